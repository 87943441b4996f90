// C-ABI entry points of the matmuls: routing between the tcgen05 kernels,
// the split-K GEMV and the general-shape CUDA-core kernels.
#include "mxb_common.cuh"
#include "mxb_internal.h"

using namespace mxb;

namespace {

constexpr size_t kAlign = 256;
size_t align_up(size_t v) { return (v + kAlign - 1) & ~(kAlign - 1); }

bool int_bits(int bits) { return bits == 1 || bits == 2 || bits == 4 || bits == 8; }
// 32: fp32 C only (no requantization; c_f32 required)
bool out_bits_ok(int bits) {
  return bits == 2 || bits == 4 || bits == 8 || bits == 16 || bits == 32;
}

}  // namespace

extern "C" {

size_t mxb_qgemm_workspace_size(int64_t M, int64_t K, int64_t N, int bits, int block) {
  if (M <= 0 || K <= 0 || N <= 0 || block <= 0) return 0;
  return align_up((size_t)M * N * sizeof(float)) + align_up(tc_qgemm_workspace(M, K, N, bits)) +
         align_up(mxb_requant_workspace_size(M * N, block));
}

size_t mxb_qgemm_kmajor_workspace_size(int64_t M, int64_t K, int64_t N, int bits, int block) {
  if (M <= 0 || K <= 0 || N <= 0 || block <= 0) return 0;
  // + the transposed scales + one byte per code of A and B (CUDA-core path)
  return mxb_qgemm_workspace_size(M, K, N, bits, block) +
         align_up((size_t)cdiv(K, block) * N * sizeof(float)) + align_up((size_t)M * K) +
         align_up((size_t)K * N);
}

}  // extern "C"

namespace {

// One implementation for both B layouts.  b_kmajor: b is B^T [N, K]
// quantized along K (K % block == 0), its scales s[n, kb].
int qgemm_impl(const void* a_packed, const float* a_scales, int64_t a_nscales,
               const void* b_packed, const float* b_scales, int64_t b_nscales, int64_t M,
               int64_t K, int64_t N, int bits, int block, int out_bits, void* c_packed,
               float* c_scales, float* c_f32, void* workspace, size_t workspace_bytes,
               bool b_kmajor, void* stream) {
  if (!int_bits(bits) || !out_bits_ok(out_bits)) return MXB_E_DTYPE;
  if (M <= 0 || K <= 0 || N <= 0 || block <= 0) return MXB_E_SHAPE;
  if (M * K >= (int64_t)1 << 31 || K * N >= (int64_t)1 << 31 || M * N >= (int64_t)1 << 31)
    return MXB_E_SHAPE;
  if (!a_packed || !a_scales || !b_packed || !b_scales) return MXB_E_ARG;
  if (out_bits == 32 ? c_f32 == nullptr : (!c_packed || !c_scales)) return MXB_E_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t kbn = cdiv(K, block);
  char* ws = static_cast<char*>(workspace);
  size_t left = workspace ? workspace_bytes : 0;
  auto take = [&](size_t bytes) -> char* {
    const size_t need = align_up(bytes);
    if (left < need) return nullptr;
    char* p = ws;
    ws += need;
    left -= need;
    return p;
  };
  bool sa_ok = a_nscales == M * kbn;
  bool sb_ok = b_nscales == kbn * N;
  const float* sb = b_scales;
  if (b_kmajor) {
    if (K % block || !sa_ok || b_nscales != N * kbn) return MXB_E_SHAPE;
    float* t = reinterpret_cast<float*>(take((size_t)kbn * N * sizeof(float)));
    if (!t) return MXB_E_WORKSPACE;
    int rc = transpose_scales(b_scales, kbn, N, t, st);
    if (rc != MXB_OK) return rc;
    sb = t;
    sb_ok = true;
  }
  const bool tc = tc_qgemm_eligible(M, K, N, bits, block, sa_ok, sb_ok, a_packed, b_packed, c_f32);
  // int16d output: the tcgen05 kernel requantizes in its epilogue
  const bool fused = tc && out_bits == 16 && ((uintptr_t)c_packed % 16) == 0;
  float* C = c_f32;
  if (C == nullptr && !fused) {
    C = reinterpret_cast<float*>(take((size_t)M * N * sizeof(float)));
    if (!C) return MXB_E_WORKSPACE;
  }
  int rc;
  if (tc) {
    const size_t need = align_up(tc_qgemm_workspace(M, K, N, bits));
    char* w = need ? take(need) : ws;
    if (need && !w) return MXB_E_WORKSPACE;
    QOut q{};
    q.count = fused ? 1 : 0;
    q.words[0] = static_cast<uint32_t*>(c_packed);
    q.scales[0] = c_scales;
    q.row_stride = (int)N;
    q.col_off = 0;
    rc = tc_qgemm(a_packed, a_scales, b_packed, sb, M, K, N, bits, block, C, &q, w, need,
                  b_kmajor, st);
  } else if (b_kmajor) {
    // CUDA-core kernel: B row-major and both operands one byte per code
    int8_t* b8 = reinterpret_cast<int8_t*>(take((size_t)K * N));
    if (!b8) return MXB_E_WORKSPACE;
    rc = widen_transpose(b_packed, K, N, bits, /*pm1*/ true, b8, st);
    if (rc != MXB_OK) return rc;
    const void* a8 = a_packed;
    if (bits != 8) {
      int8_t* w = reinterpret_cast<int8_t*>(take((size_t)M * K));
      if (!w) return MXB_E_WORKSPACE;
      rc = widen_codes(a_packed, M * K, bits, w, /*pm1*/ true, st);
      if (rc != MXB_OK) return rc;
      a8 = w;
    }
    rc = qgemm_generic(a8, a_scales, true, b8, sb, true, M, K, N, 8, block, C, st);
  } else {
    rc = qgemm_generic(a_packed, a_scales, sa_ok, b_packed, b_scales, sb_ok, M, K, N, bits,
                       block, C, st);
  }
  if (rc != MXB_OK || out_bits == 32 || fused) return rc;
  return mxb_requant_f32(C, M * N, block, out_bits, c_packed, c_scales, left ? ws : nullptr,
                         left, st);
}

}  // namespace

extern "C" {

int mxb_qgemm(const void* a_packed, const float* a_scales, int64_t a_nscales,
              const void* b_packed, const float* b_scales, int64_t b_nscales, int64_t M,
              int64_t K, int64_t N, int bits, int block, int out_bits, void* c_packed,
              float* c_scales, float* c_f32, void* workspace, size_t workspace_bytes,
              void* stream) {
  return qgemm_impl(a_packed, a_scales, a_nscales, b_packed, b_scales, b_nscales, M, K, N, bits,
                    block, out_bits, c_packed, c_scales, c_f32, workspace, workspace_bytes,
                    false, stream);
}

int mxb_qgemm_kmajor(const void* a_packed, const float* a_scales, int64_t a_nscales,
                     const void* bt_packed, const float* bt_scales, int64_t bt_nscales,
                     int64_t M, int64_t K, int64_t N, int bits, int block, int out_bits,
                     void* c_packed, float* c_scales, float* c_f32, void* workspace,
                     size_t workspace_bytes, void* stream) {
  return qgemm_impl(a_packed, a_scales, a_nscales, bt_packed, bt_scales, bt_nscales, M, K, N,
                    bits, block, out_bits, c_packed, c_scales, c_f32, workspace,
                    workspace_bytes, true, stream);
}

static int qgemm_sharded_impl(const void* a_packed, const float* a_scales, int64_t a_nscales,
                              const void* b_packed, const float* b_scales, int64_t b_nscales,
                              int64_t M, int64_t K, int64_t N_local, int bits, int block,
                              int64_t N_full, int64_t n_off, int nranks,
                              void* const* out_words, float* const* out_scales,
                              void* const* sync_blocks, int rank, void* workspace,
                              size_t workspace_bytes, void* stream);

int mxb_qgemm_sharded(const void* a_packed, const float* a_scales, int64_t a_nscales,
                      const void* b_packed, const float* b_scales, int64_t b_nscales,
                      int64_t M, int64_t K, int64_t N_local, int bits, int block,
                      int64_t N_full, int64_t n_off, int nranks, void* const* out_words,
                      float* const* out_scales, void* workspace, size_t workspace_bytes,
                      void* stream) {
  return qgemm_sharded_impl(a_packed, a_scales, a_nscales, b_packed, b_scales, b_nscales, M, K,
                            N_local, bits, block, N_full, n_off, nranks, out_words, out_scales,
                            nullptr, 0, workspace, workspace_bytes, stream);
}

int mxb_qgemm_sharded_sync(const void* a_packed, const float* a_scales, int64_t a_nscales,
                           const void* b_packed, const float* b_scales, int64_t b_nscales,
                           int64_t M, int64_t K, int64_t N_local, int bits, int block,
                           int64_t N_full, int64_t n_off, int nranks, int rank,
                           void* const* out_words, float* const* out_scales,
                           void* const* sync_blocks, void* workspace, size_t workspace_bytes,
                           void* stream) {
  if (!sync_blocks || rank < 0 || rank >= nranks) return MXB_E_ARG;
  return qgemm_sharded_impl(a_packed, a_scales, a_nscales, b_packed, b_scales, b_nscales, M, K,
                            N_local, bits, block, N_full, n_off, nranks, out_words, out_scales,
                            sync_blocks, rank, workspace, workspace_bytes, stream);
}

static int qgemm_sharded_impl(const void* a_packed, const float* a_scales, int64_t a_nscales,
                              const void* b_packed, const float* b_scales, int64_t b_nscales,
                              int64_t M, int64_t K, int64_t N_local, int bits, int block,
                              int64_t N_full, int64_t n_off, int nranks,
                              void* const* out_words, float* const* out_scales,
                              void* const* sync_blocks, int rank, void* workspace,
                              size_t workspace_bytes, void* stream) {
  if (!int_bits(bits)) return MXB_E_DTYPE;
  if (M <= 0 || K <= 0 || N_local <= 0 || block <= 0) return MXB_E_SHAPE;
  if (nranks < 1 || nranks > kMaxPeers || !out_words || !out_scales) return MXB_E_ARG;
  if (N_full % 128 || n_off % 128 || n_off < 0 || n_off + N_local > N_full) return MXB_E_SHAPE;
  if (M * K >= (int64_t)1 << 31 || K * N_local >= (int64_t)1 << 31 ||
      M * N_full >= (int64_t)1 << 31)
    return MXB_E_SHAPE;
  if (!a_packed || !a_scales || !b_packed || !b_scales) return MXB_E_ARG;
  const int64_t kbn = cdiv(K, block);
  const bool sa_ok = a_nscales == M * kbn, sb_ok = b_nscales == kbn * N_local;
  // the fused epilogue writes C only as int16d codes, so C itself is not needed
  if (!tc_qgemm_eligible(M, K, N_local, bits, block, sa_ok, sb_ok, a_packed, b_packed, nullptr))
    return MXB_E_SHAPE;
  QOut q{};
  q.count = nranks;
  q.row_stride = (int)N_full;
  q.col_off = (int)n_off;
  for (int r = 0; r < nranks; ++r) {
    if (!out_words[r] || !out_scales[r] || ((uintptr_t)out_words[r] & 15)) return MXB_E_ARG;
    q.words[r] = static_cast<uint32_t*>(out_words[r]);
    q.scales[r] = out_scales[r];
    if (sync_blocks) {
      if (!sync_blocks[r] || ((uintptr_t)sync_blocks[r] & 7)) return MXB_E_ARG;
      q.sync[r] = static_cast<unsigned long long*>(sync_blocks[r]);
    }
  }
  q.rank = rank;
  const size_t need = align_up(tc_qgemm_workspace(M, K, N_local, bits));
  if (need && (!workspace || workspace_bytes < need)) return MXB_E_WORKSPACE;
  return tc_qgemm(a_packed, a_scales, b_packed, b_scales, M, K, N_local, bits, block, nullptr,
                  &q, workspace, need, false, static_cast<cudaStream_t>(stream));
}

int mxb_peer_barrier(int nranks, int rank, void* const* sync_blocks, void* stream) {
  if (nranks < 1 || nranks > kMaxPeers || rank < 0 || rank >= nranks || !sync_blocks)
    return MXB_E_ARG;
  unsigned long long* sync[kMaxPeers] = {};
  for (int r = 0; r < nranks; ++r) {
    if (!sync_blocks[r] || ((uintptr_t)sync_blocks[r] & 7)) return MXB_E_ARG;
    sync[r] = static_cast<unsigned long long*>(sync_blocks[r]);
  }
  return peer_barrier(sync, nranks, rank, static_cast<cudaStream_t>(stream));
}

size_t mxb_linear_wonly_workspace_size(int64_t M, int64_t K, int64_t N, int bits, int kind,
                                       int block, int mode) {
  (void)mode;
  if (M <= 0 || K <= 0 || N <= 0) return 0;
  GemvPlan p = gemv_plan(M, K, N, bits, kind, block, nullptr, nullptr, -1, nullptr);
  return p.ok ? p.ws_bytes : 0;
}

int mxb_linear_wonly(const void* x, int x_dtype, int64_t M, int64_t K, const void* w_packed,
                     const float* w_scales, int64_t N, int bits, int kind, int block, int mode,
                     float* y, void* workspace, size_t workspace_bytes, void* stream) {
  if (kind == MXB_KIND_FLOAT ? bits != 4 : !int_bits(bits)) return MXB_E_DTYPE;
  if (kind != MXB_KIND_INT && kind != MXB_KIND_FLOAT) return MXB_E_DTYPE;
  if (x_dtype != MXB_F32 && x_dtype != MXB_BF16) return MXB_E_DTYPE;
  if (mode != MXB_MODE_PARITY && mode != MXB_MODE_FAST) return MXB_E_ARG;
  if (M < 0 || K <= 0 || N <= 0 || block <= 0) return MXB_E_SHAPE;
  if (M == 0) return MXB_OK;
  if (M * K >= (int64_t)1 << 31 || K * N >= (int64_t)1 << 31 || M * N >= (int64_t)1 << 31)
    return MXB_E_SHAPE;
  if (!x || !w_packed || !w_scales || !y) return MXB_E_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  GemvPlan p = gemv_plan(M, K, N, bits, kind, block, w_packed, y, x_dtype, x);
  if (p.ok) {
    if (!workspace || workspace_bytes < p.ws_bytes) return MXB_E_WORKSPACE;
    return gemv_run(p, x, x_dtype, M, K, w_packed, w_scales, N, bits, kind, block, y,
                    static_cast<float*>(workspace), st);
  }
  if (tc_wonly_eligible(x, x_dtype, M, K, w_packed, N, bits, kind, block, y))
    return tc_wonly(x, M, K, w_packed, w_scales, N, bits, kind, block, mode, y, st);
  return wonly_generic(x, x_dtype, M, K, w_packed, w_scales, N, bits, kind, block, y, st);
}

int mxb_linear_wonly_kmajor(const void* x, int x_dtype, int64_t M, int64_t K,
                            const void* w_packed, const float* w_scales, int64_t N, int bits,
                            int kind, int block, int mode, float* y, void* stream) {
  if (kind == MXB_KIND_FLOAT ? bits != 4 : !int_bits(bits)) return MXB_E_DTYPE;
  if (kind != MXB_KIND_INT && kind != MXB_KIND_FLOAT) return MXB_E_DTYPE;
  if (x_dtype != MXB_F32 && x_dtype != MXB_BF16) return MXB_E_DTYPE;
  if (mode != MXB_MODE_PARITY && mode != MXB_MODE_FAST) return MXB_E_ARG;
  if (M < 0 || K <= 0 || N <= 0 || block <= 0) return MXB_E_SHAPE;
  if (M == 0) return MXB_OK;
  if (M * K >= (int64_t)1 << 31 || K * N >= (int64_t)1 << 31 || M * N >= (int64_t)1 << 31)
    return MXB_E_SHAPE;
  if (!x || !w_packed || !w_scales || !y) return MXB_E_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (tc_wonly_eligible(x, x_dtype, M, K, w_packed, N, bits, kind, block, y, /*kmajor*/ true))
    return tc_wonly(x, M, K, w_packed, w_scales, N, bits, kind, block, mode, y, st, true);
  return wonly_generic(x, x_dtype, M, K, w_packed, w_scales, N, bits, kind, block, y, st, true);
}

}  // extern "C"
