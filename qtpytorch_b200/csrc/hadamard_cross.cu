// Cross-shard stage of a row Walsh-Hadamard transform whose columns are
// split over G ranks, fused with the reorder of the all-gathered shards.
//
// With N = G * L and column j = g * L + l, the Sylvester matrix factors as
// H_N = H_G (x) H_L, so the unrotation of a row (hadamard_rotation.unrotate,
// mxtorch.py:2892-2904: y -> WHT(y) / sqrt(N) * signs) splits into
//   t_g = WHT_L(y_g) / sqrt(L)            on each rank's own columns, then
//   z[g*L + l] = (sum_h H_G[g, h] t_h[l]) / sqrt(G) * signs[g*L + l]
// after the all-gather.  This kernel is the second line: it reads the
// gathered [G][M][L] buffer (rank-major, as NCCL leaves it), runs the
// G-point butterflies (largest stride first) and writes row-major [M][N].
// The rounding differs from the unsplit transform by a few fp32 ulps of
// the row's magnitude (stage order), inside the linear's 1e-5 bound.
#include "mxb_common.cuh"
#include "mxb_internal.h"

using namespace mxb;

namespace {

template <int G>
__global__ void __launch_bounds__(256) hcross_kernel(const float4* __restrict__ t, int64_t M,
                                                     int64_t L4, float rsq_div,
                                                     const float4* __restrict__ signs,
                                                     float4* __restrict__ out) {
  const int64_t total = M * L4;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = i / L4, l4 = i % L4;
    float4 v[G];
#pragma unroll
    for (int g = 0; g < G; ++g) v[g] = __ldcs(t + ((int64_t)g * M + m) * L4 + l4);
#pragma unroll
    for (int h = G / 2; h >= 1; h /= 2) {
#pragma unroll
      for (int g = 0; g < G; ++g) {
        if (g & h) continue;
        const float4 e = v[g], o = v[g + h];
        v[g] = make_float4(__fadd_rn(e.x, o.x), __fadd_rn(e.y, o.y), __fadd_rn(e.z, o.z),
                           __fadd_rn(e.w, o.w));
        v[g + h] = make_float4(__fsub_rn(e.x, o.x), __fsub_rn(e.y, o.y), __fsub_rn(e.z, o.z),
                               __fsub_rn(e.w, o.w));
      }
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float4 s = __ldg(signs + (int64_t)g * L4 + l4);
      float4 r = v[g];
      if (G > 1) {
        r.x = __fdiv_rn(r.x, rsq_div);
        r.y = __fdiv_rn(r.y, rsq_div);
        r.z = __fdiv_rn(r.z, rsq_div);
        r.w = __fdiv_rn(r.w, rsq_div);
      }
      out[m * (G * L4) + (int64_t)g * L4 + l4] =
          make_float4(__fmul_rn(r.x, s.x), __fmul_rn(r.y, s.y), __fmul_rn(r.z, s.z),
                      __fmul_rn(r.w, s.w));
    }
  }
}

template <int G>
int launch(const float* t, int64_t M, int64_t L, const float* signs, float* out,
           cudaStream_t st) {
  const int64_t L4 = L / 4;
  int64_t blocks = cdiv(M * L4, 256);
  if (blocks > (int64_t)kSMs * 16) blocks = (int64_t)kSMs * 16;
  hcross_kernel<G><<<(unsigned)blocks, 256, 0, st>>>(
      reinterpret_cast<const float4*>(t), M, L4, (float)sqrt((double)G),
      reinterpret_cast<const float4*>(signs), reinterpret_cast<float4*>(out));
  MXB_LAUNCH_CHECK();
  return MXB_OK;
}

}  // namespace

extern "C" int mxb_hadamard_cross(const float* t, int64_t M, int64_t L, int G,
                                  const float* signs, float* out, void* stream) {
  if (M < 0 || L <= 0 || L % 4) return MXB_E_SHAPE;
  if (M == 0) return MXB_OK;
  if (!t || !signs || !out) return MXB_E_ARG;
  if ((((uintptr_t)t) | ((uintptr_t)signs) | ((uintptr_t)out)) & 15) return MXB_E_ALIGN;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (G) {
    case 1: return launch<1>(t, M, L, signs, out, st);
    case 2: return launch<2>(t, M, L, signs, out, st);
    case 4: return launch<4>(t, M, L, signs, out, st);
    case 8: return launch<8>(t, M, L, signs, out, st);
  }
  return MXB_E_SHAPE;
}
