// CUDA-core matmul kernels: the general-shape packed integer GEMM, the
// general-shape weight-only GEMM and the split-K decode GEMV.
//
// The tcgen05 kernels (gemm_tc.cu) take the aligned large shapes; these
// cover everything else with the same arithmetic contract.
#include "mxb_common.cuh"
#include "mxb_internal.h"

using namespace mxb;

namespace {

// Sign-extended integer code of element e of a packed stream.
template <int BITS>
__device__ __forceinline__ int icode(const uint8_t* __restrict__ p, int64_t e) {
  if constexpr (BITS == 8) {
    return (int)(int8_t)__ldg(p + e);
  } else {
    constexpr int PER = 8 / BITS;
    uint32_t b = __ldg(p + e / PER);
    return sext((b >> ((e % PER) * BITS)) & ((1u << BITS) - 1u), BITS);
  }
}

// ── packed integer GEMM, any shape ───────────────────────────────────────────
// 64x64 output tile per CTA, 256 threads, 4x4 outputs per thread.  K runs in
// chunks of <= 32 inside each scale block; int32 partials are promoted into
// the fp32 accumulator once per K-block, in K-block order.
constexpr int GT = 64, GK = 32;

template <int BITS>
__global__ void __launch_bounds__(256) qgemm_generic_kernel(
    const uint8_t* __restrict__ A, const float* __restrict__ sa, bool sa_ok,
    const uint8_t* __restrict__ B, const float* __restrict__ sb, bool sb_ok, int M, int K,
    int N, int block, float* __restrict__ C) {
  __shared__ int As[GK][GT + 1];
  __shared__ int Bs[GK][GT + 1];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int m0 = blockIdx.y * GT, n0 = blockIdx.x * GT;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;
  const int kbn = (K + block - 1) / block;
  for (int kb = 0; kb < kbn; ++kb) {
    const int k0 = kb * block, k1 = min(k0 + block, K);
    int part[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) part[i][j] = 0;
    for (int kc = k0; kc < k1; kc += GK) {
      const int kn = min(GK, k1 - kc);
      __syncthreads();
      for (int idx = threadIdx.x; idx < GK * GT; idx += 256) {
        int kk = idx / GT, c = idx % GT;
        int m = m0 + c, n = n0 + c, k = kc + kk;
        As[kk][c] = (kk < kn && m < M) ? icode<BITS>(A, (int64_t)m * K + k) : 0;
        Bs[kk][c] = (kk < kn && n < N) ? icode<BITS>(B, (int64_t)k * N + n) : 0;
      }
      __syncthreads();
      for (int kk = 0; kk < kn; ++kk) {
        int a[4], b[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
        for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tx * 4 + j];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) part[i][j] += a[i] * b[j];
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int m = m0 + ty * 4 + i;
      const float s_a = (sa_ok && m < M) ? __ldg(sa + (int64_t)m * kbn + kb) : 1.0f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int n = n0 + tx * 4 + j;
        const float s_b = (sb_ok && n < N) ? __ldg(sb + (int64_t)kb * N + n) : 1.0f;
        // C += (P * sa) * sb, each step one fp32 rounding (mxtorch.py:1366)
        acc[i][j] = __fadd_rn(acc[i][j], __fmul_rn(__fmul_rn((float)part[i][j], s_a), s_b));
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int m = m0 + ty * 4 + i;
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + tx * 4 + j;
      if (n < N) C[(int64_t)m * N + n] = acc[i][j];
    }
  }
}

// ── weight-only GEMM, any shape (fp32 FMA) ───────────────────────────────────
// KMAJ: the weight is W [N, K] quantized flat (element (k, n) at n * K + k,
// the layout of mx_dynamic_linear's weight) instead of W^T [K, N].
template <int BITS, int KIND, bool KMAJ, typename XT>
__global__ void __launch_bounds__(256) wonly_generic_kernel(
    const XT* __restrict__ x, int M, int K, const uint8_t* __restrict__ W,
    const float* __restrict__ ws, int N, int block, float* __restrict__ y) {
  __shared__ float Xs[GK][GT + 1];
  __shared__ float Ws[GK][GT + 1];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int m0 = blockIdx.y * GT, n0 = blockIdx.x * GT;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;
  for (int kc = 0; kc < K; kc += GK) {
    __syncthreads();
    for (int idx = threadIdx.x; idx < GK * GT; idx += 256) {
      int kk = idx / GT, c = idx % GT, k = kc + kk;
      int m = m0 + c, n = n0 + c;
      Xs[kk][c] = (k < K && m < M) ? load_as_f32(x, (int64_t)m * K + k) : 0.0f;
      float w = 0.0f;
      if (k < K && n < N) {
        const int64_t e = KMAJ ? (int64_t)n * K + k : (int64_t)k * N + n;
        uint32_t raw;
        if constexpr (BITS == 8) {
          raw = __ldg(W + e);
        } else {
          constexpr int PER = 8 / BITS;
          raw = (__ldg(W + e / PER) >> ((e % PER) * BITS)) & ((1u << BITS) - 1u);
        }
        w = dequant_code<BITS, KIND>(raw, __ldg(ws + e / block));
      }
      Ws[kk][c] = w;
    }
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < GK; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = Xs[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = Ws[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int m = m0 + ty * 4 + i;
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + tx * 4 + j;
      if (n < N) y[(int64_t)m * N + n] = acc[i][j];
    }
  }
}

}  // namespace

namespace mxb {

int qgemm_generic(const void* a, const float* sa, bool sa_ok, const void* b, const float* sb,
                  bool sb_ok, int64_t M, int64_t K, int64_t N, int bits, int block, float* C,
                  cudaStream_t st) {
  dim3 grid((unsigned)cdiv(N, GT), (unsigned)cdiv(M, GT));
  const uint8_t* A = static_cast<const uint8_t*>(a);
  const uint8_t* B = static_cast<const uint8_t*>(b);
  switch (bits) {
    case 1: qgemm_generic_kernel<1><<<grid, 256, 0, st>>>(A, sa, sa_ok, B, sb, sb_ok, (int)M, (int)K, (int)N, block, C); break;
    case 2: qgemm_generic_kernel<2><<<grid, 256, 0, st>>>(A, sa, sa_ok, B, sb, sb_ok, (int)M, (int)K, (int)N, block, C); break;
    case 4: qgemm_generic_kernel<4><<<grid, 256, 0, st>>>(A, sa, sa_ok, B, sb, sb_ok, (int)M, (int)K, (int)N, block, C); break;
    case 8: qgemm_generic_kernel<8><<<grid, 256, 0, st>>>(A, sa, sa_ok, B, sb, sb_ok, (int)M, (int)K, (int)N, block, C); break;
    default: return MXB_E_DTYPE;
  }
  MXB_LAUNCH_CHECK();
  return MXB_OK;
}

template <bool KMAJ, typename XT>
static int wonly_generic_t(const XT* x, int64_t M, int64_t K, const uint8_t* W, const float* ws,
                           int64_t N, int bits, int kind, int block, float* y, cudaStream_t st) {
  dim3 grid((unsigned)cdiv(N, GT), (unsigned)cdiv(M, GT));
  const int iM = (int)M, iK = (int)K, iN = (int)N;
  if (kind == MXB_KIND_FLOAT) {
    wonly_generic_kernel<4, MXB_KIND_FLOAT, KMAJ, XT><<<grid, 256, 0, st>>>(x, iM, iK, W, ws, iN, block, y);
  } else {
    switch (bits) {
      case 1: wonly_generic_kernel<1, MXB_KIND_INT, KMAJ, XT><<<grid, 256, 0, st>>>(x, iM, iK, W, ws, iN, block, y); break;
      case 2: wonly_generic_kernel<2, MXB_KIND_INT, KMAJ, XT><<<grid, 256, 0, st>>>(x, iM, iK, W, ws, iN, block, y); break;
      case 4: wonly_generic_kernel<4, MXB_KIND_INT, KMAJ, XT><<<grid, 256, 0, st>>>(x, iM, iK, W, ws, iN, block, y); break;
      case 8: wonly_generic_kernel<8, MXB_KIND_INT, KMAJ, XT><<<grid, 256, 0, st>>>(x, iM, iK, W, ws, iN, block, y); break;
      default: return MXB_E_DTYPE;
    }
  }
  MXB_LAUNCH_CHECK();
  return MXB_OK;
}

int wonly_generic(const void* x, int x_dtype, int64_t M, int64_t K, const void* w,
                  const float* ws, int64_t N, int bits, int kind, int block, float* y,
                  cudaStream_t st, bool kmajor) {
  const uint8_t* W = static_cast<const uint8_t*>(w);
  if (x_dtype == MXB_F32) {
    const float* xf = static_cast<const float*>(x);
    return kmajor ? wonly_generic_t<true>(xf, M, K, W, ws, N, bits, kind, block, y, st)
                  : wonly_generic_t<false>(xf, M, K, W, ws, N, bits, kind, block, y, st);
  }
  if (x_dtype == MXB_BF16) {
    const __nv_bfloat16* xb = static_cast<const __nv_bfloat16*>(x);
    return kmajor ? wonly_generic_t<true>(xb, M, K, W, ws, N, bits, kind, block, y, st)
                  : wonly_generic_t<false>(xb, M, K, W, ws, N, bits, kind, block, y, st);
  }
  return MXB_E_DTYPE;
}

}  // namespace mxb
