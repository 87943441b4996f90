// Internal entry points shared between the library's translation units.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

// quantize.cu
int mxb_requant_f32(const float* c, int64_t n, int block, int out_bits, void* packed,
                    float* scales, void* ws, size_t wsb, cudaStream_t st);
size_t mxb_requant_workspace_size(int64_t n, int block);

namespace mxb {

// gemm_cuda_core.cu
int qgemm_generic(const void* a, const float* sa, bool sa_ok, const void* b, const float* sb,
                  bool sb_ok, int64_t M, int64_t K, int64_t N, int bits, int block, float* C,
                  cudaStream_t st);
// kmajor: the weight is W [N, K] quantized flat instead of W^T [K, N]
int wonly_generic(const void* x, int x_dtype, int64_t M, int64_t K, const void* w,
                  const float* ws, int64_t N, int bits, int kind, int block, float* y,
                  cudaStream_t st, bool kmajor = false);

// gemv.cu
constexpr int kDecMaxKc = 2048;  // K rows per CTA of the tcgen05 decode kernel
struct GemvPlan {
  bool ok;          // shape/alignment supported by the split-K kernel
  int splits;       // K splits
  int krows;        // rows of K per split
  size_t ws_bytes;  // partial-sum workspace
  int kernel = 0;   // 0: 8 columns per thread, any code width; 1: wide loads (int4/int8);
                    // 4: tcgen05 decode kernel (bf16 x, integer codes, 3 <= M <= 32)
  int lb = 0;       // kernel 1: code bytes per thread and row (4, 8 or 16)
  int max_krows = 0;  // largest rows per split the kernel accepts
};
// x_dtype < 0: the dtype is not known yet (workspace queries); the plan then
// covers the largest workspace either activation dtype may need.
GemvPlan gemv_plan(int64_t M, int64_t K, int64_t N, int bits, int kind, int block,
                   const void* w, const void* y, int x_dtype, const void* x);
int gemv_run(const GemvPlan& plan, const void* x, int x_dtype, int64_t M, int64_t K,
             const void* w, const float* ws, int64_t N, int bits, int kind, int block,
             float* y, float* partial, cudaStream_t st);

// gemm_tc.cu (tcgen05)
constexpr int kMaxPeers = 8;
// int16d outputs of the int8 GEMM's fused requantization: `count` buffers
// written with the same codes and scales (one for a plain matmul; every
// rank's full-width output for a column-sharded one), rows of `row_stride`
// columns, this launch's columns starting at `col_off`.
struct QOut {
  uint32_t* words[kMaxPeers];
  float* scales[kMaxPeers];
  int count;
  int row_stride;
  int col_off;
  // completion barrier across the ranks after the kernel (sync[0] != null):
  // sync[r] is rank r's barrier block, this rank's own included; `rank`
  // indexes this rank
  unsigned long long* sync[kMaxPeers];
  int rank;
};
// Device address of the library's device error word (mxb_device_error), for
// kernels outside gemm_tc.cu; nullptr if the lookup fails.
int* device_error_ptr();
// The cross-rank barrier kernel alone, on stream st (same counters as the
// barrier that follows a sharded matmul).
int peer_barrier(unsigned long long* const* sync, int nranks, int rank, cudaStream_t st);
// Layout of a rank's barrier block (zeroed once by the caller): [1] this
// rank's call counter, [8 + r] the call counter rank r last signalled to
// this rank.
constexpr int kSyncWords = 16;
bool tc_qgemm_eligible(int64_t M, int64_t K, int64_t N, int bits, int block, bool sa_ok,
                       bool sb_ok, const void* a, const void* b, const float* c);
size_t tc_qgemm_workspace(int64_t M, int64_t K, int64_t N, int bits);
int tc_qgemm(const void* a, const float* sa, const void* b, const float* sb, int64_t M,
             int64_t K, int64_t N, int bits, int block, float* C, const QOut* qout, void* ws,
             size_t wsb, bool b_kmajor, cudaStream_t st);
// (b_kmajor also gives 1-bit codes their +-1 meaning)
// layout helpers of the k-major matmul
int transpose_scales(const float* s, int64_t kbn, int64_t N, float* out, cudaStream_t st);
// pm1: 1-bit codes as +-1 (their dequantized meaning) instead of 0 / -1
int widen_transpose(const void* bt, int64_t K, int64_t N, int bits, bool pm1, int8_t* out,
                    cudaStream_t st);
int widen_codes(const void* p, int64_t n, int bits, int8_t* out, bool pm1, cudaStream_t st);
// kmajor: W [N, K] quantized flat (scale s[n, k / block]) instead of W^T [K, N]
bool tc_wonly_eligible(const void* x, int x_dtype, int64_t M, int64_t K, const void* w,
                       int64_t N, int bits, int kind, int block, const float* y,
                       bool kmajor = false);
int tc_wonly(const void* x, int64_t M, int64_t K, const void* w, const float* ws, int64_t N,
             int bits, int kind, int block, int mode, float* y, cudaStream_t st,
             bool kmajor = false);
bool tc_dec_eligible(const void* x, int x_dtype, int64_t M, int64_t K, const void* w, int64_t N,
                     int bits, int kind, int block);
void tc_dec_plan(int64_t M, int64_t K, int64_t N, int* splits, int* kc);
int tc_wonly_dec(const void* x, int64_t M, int64_t K, const void* w, const float* ws, int64_t N,
                 int bits, int block, int kc, int splits, float* out, cudaStream_t st);
}  // namespace mxb
