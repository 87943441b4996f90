// Split-K GEMV for the decode regime of the weight-only linear (M <= 16).
//
// y[m, n] = sum_k x[m, k] * fl(code[k, n] * s[k, n / block])   (mxtorch.py:7454-7473)
//
// The weight stream dominates the traffic, so the kernel is HBM-bound: each
// thread owns 8 adjacent output columns and walks a slice of K, loading the
// 8 codes of one row with one load (one warp reads 32 * bits bytes per row,
// contiguous); x for the slice is staged in shared memory as fp32.  Each K
// split writes its own partial sums; a second kernel adds the splits in a
// fixed order, so results are deterministic.
#include "mxb_common.cuh"
#include "mxb_internal.h"

using namespace mxb;

namespace {

constexpr int kThreads = 128;       // threads per CTA
constexpr int kCols = 8;            // output columns per thread
constexpr int kMaxRows = 256;       // K rows per split (shared x slice)
constexpr int kCtaCols = kThreads * kCols;

template <int BITS>
__device__ __forceinline__ uint64_t load_codes(const uint8_t* p) {
  if constexpr (BITS == 8) {
    uint2 v = __ldcs(reinterpret_cast<const uint2*>(p));
    return (uint64_t)v.x | ((uint64_t)v.y << 32);
  } else if constexpr (BITS == 4) {
    return __ldcs(reinterpret_cast<const uint32_t*>(p));
  } else if constexpr (BITS == 2) {
    return __ldcs(reinterpret_cast<const uint16_t*>(p));
  } else {
    return __ldcs(p);
  }
}

template <int BITS, int KIND, int MT, typename XT>
__global__ void __launch_bounds__(kThreads) gemv_kernel(const XT* __restrict__ x, int M, int K,
                                                        const uint8_t* __restrict__ W,
                                                        const float* __restrict__ ws, int N,
                                                        int block, int krows,
                                                        float* __restrict__ part) {
  __shared__ float xs[MT][kMaxRows];
  const int k0 = blockIdx.y * krows;
  const int kn = min(krows, K - k0);
  for (int i = threadIdx.x; i < MT * kMaxRows; i += kThreads) {
    int m = i / kMaxRows, kk = i % kMaxRows;
    xs[m][kk] = (m < M && kk < kn) ? load_as_f32(x, (int64_t)m * K + k0 + kk) : 0.0f;
  }
  __syncthreads();
  const int c0 = (blockIdx.x * kThreads + threadIdx.x) * kCols;
  if (c0 >= N) return;
  float acc[MT][kCols];
#pragma unroll
  for (int m = 0; m < MT; ++m)
#pragma unroll
    for (int c = 0; c < kCols; ++c) acc[m][c] = 0.0f;

  const int64_t row_bytes = (int64_t)N * BITS / 8;
  const int64_t nsb = N / block;
  const uint8_t* wp = W + (int64_t)k0 * row_bytes + (int64_t)c0 * BITS / 8;
  const float* sp = ws + (int64_t)k0 * nsb + c0 / block;
#pragma unroll 8
  for (int kk = 0; kk < kn; ++kk) {
    const uint64_t word = load_codes<BITS>(wp + kk * row_bytes);
    const float s = __ldg(sp + kk * nsb);
    float w[kCols];
#pragma unroll
    for (int c = 0; c < kCols; ++c)
      w[c] = dequant_code<BITS, KIND>((uint32_t)(word >> (c * BITS)) & ((1u << BITS) - 1u), s);
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      const float xv = xs[m][kk];
#pragma unroll
      for (int c = 0; c < kCols; ++c) acc[m][c] = fmaf(xv, w[c], acc[m][c]);
    }
  }
  float* out = part + (int64_t)blockIdx.y * M * N + c0;
#pragma unroll
  for (int m = 0; m < MT; ++m) {
    if (m < M) {
      float4* o = reinterpret_cast<float4*>(out + (int64_t)m * N);
      o[0] = make_float4(acc[m][0], acc[m][1], acc[m][2], acc[m][3]);
      o[1] = make_float4(acc[m][4], acc[m][5], acc[m][6], acc[m][7]);
    }
  }
}

__global__ void __launch_bounds__(256) split_reduce_kernel(const float* __restrict__ part,
                                                           int splits, int64_t mn,
                                                           float* __restrict__ y) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < mn;
       i += (int64_t)gridDim.x * blockDim.x) {
    float s = 0.0f;
    for (int j = 0; j < splits; ++j) s = __fadd_rn(s, part[(int64_t)j * mn + i]);
    y[i] = s;
  }
}

template <int BITS, int KIND, typename XT>
int launch_mt(int mt, dim3 grid, const XT* x, int M, int K, const uint8_t* W, const float* ws,
              int N, int block, int krows, float* part, cudaStream_t st) {
  switch (mt) {
    case 1: gemv_kernel<BITS, KIND, 1, XT><<<grid, kThreads, 0, st>>>(x, M, K, W, ws, N, block, krows, part); break;
    case 2: gemv_kernel<BITS, KIND, 2, XT><<<grid, kThreads, 0, st>>>(x, M, K, W, ws, N, block, krows, part); break;
    case 4: gemv_kernel<BITS, KIND, 4, XT><<<grid, kThreads, 0, st>>>(x, M, K, W, ws, N, block, krows, part); break;
    case 8: gemv_kernel<BITS, KIND, 8, XT><<<grid, kThreads, 0, st>>>(x, M, K, W, ws, N, block, krows, part); break;
    default: gemv_kernel<BITS, KIND, 16, XT><<<grid, kThreads, 0, st>>>(x, M, K, W, ws, N, block, krows, part); break;
  }
  MXB_LAUNCH_CHECK();
  return MXB_OK;
}

template <typename XT>
int launch_t(int mt, dim3 grid, const XT* x, int M, int K, const uint8_t* W, const float* ws,
             int N, int bits, int kind, int block, int krows, float* part, cudaStream_t st) {
  if (kind == MXB_KIND_FLOAT)
    return launch_mt<4, MXB_KIND_FLOAT>(mt, grid, x, M, K, W, ws, N, block, krows, part, st);
  switch (bits) {
    case 1: return launch_mt<1, MXB_KIND_INT>(mt, grid, x, M, K, W, ws, N, block, krows, part, st);
    case 2: return launch_mt<2, MXB_KIND_INT>(mt, grid, x, M, K, W, ws, N, block, krows, part, st);
    case 4: return launch_mt<4, MXB_KIND_INT>(mt, grid, x, M, K, W, ws, N, block, krows, part, st);
    case 8: return launch_mt<8, MXB_KIND_INT>(mt, grid, x, M, K, W, ws, N, block, krows, part, st);
  }
  return MXB_E_DTYPE;
}

}  // namespace

namespace mxb {

GemvPlan gemv_plan(int64_t M, int64_t K, int64_t N, int bits, int kind, int block,
                   const void* w, const void* y) {
  GemvPlan p{false, 0, 0, 0};
  if (M < 1 || M > 16 || K < 1 || N < kCols) return p;
  if (N % kCols || block % kCols || N % block) return p;
  if (((uintptr_t)w % (uintptr_t)bits) || ((uintptr_t)y % 16)) return p;
  (void)kind;
  const int64_t groups = cdiv(N, kCtaCols);
  int64_t splits = cdiv(4 * kSMs, groups);
  int64_t krows = cdiv(cdiv(K, splits), 8) * 8;
  if (krows > kMaxRows) krows = kMaxRows;
  if (krows < 8) krows = 8;
  splits = cdiv(K, krows);
  p.ok = true;
  p.splits = (int)splits;
  p.krows = (int)krows;
  p.ws_bytes = (size_t)splits * M * N * sizeof(float);
  return p;
}

int gemv_run(const GemvPlan& plan, const void* x, int x_dtype, int64_t M, int64_t K,
             const void* w, const float* ws, int64_t N, int bits, int kind, int block,
             float* y, float* partial, cudaStream_t st) {
  const int mt = M <= 1 ? 1 : M <= 2 ? 2 : M <= 4 ? 4 : M <= 8 ? 8 : 16;
  dim3 grid((unsigned)cdiv(N, kCtaCols), (unsigned)plan.splits);
  const uint8_t* W = static_cast<const uint8_t*>(w);
  int rc;
  if (x_dtype == MXB_F32)
    rc = launch_t(mt, grid, static_cast<const float*>(x), (int)M, (int)K, W, ws, (int)N, bits,
                  kind, block, plan.krows, partial, st);
  else if (x_dtype == MXB_BF16)
    rc = launch_t(mt, grid, static_cast<const __nv_bfloat16*>(x), (int)M, (int)K, W, ws,
                  (int)N, bits, kind, block, plan.krows, partial, st);
  else
    return MXB_E_DTYPE;
  if (rc != MXB_OK) return rc;
  const int64_t mn = M * N;
  int64_t g = cdiv(mn, 256);
  if (g > kSMs * 8) g = kSMs * 8;
  split_reduce_kernel<<<(unsigned)g, 256, 0, st>>>(partial, plan.splits, mn, y);
  MXB_LAUNCH_CHECK();
  return MXB_OK;
}

}  // namespace mxb
