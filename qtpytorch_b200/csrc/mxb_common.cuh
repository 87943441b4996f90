// Shared definitions for the mxb CUDA library (sm_100a only).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "../../include/mxb.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "mxb is built for sm_100a only"
#endif

#define MXB_CUDA_TRY(expr)                                 \
  do {                                                     \
    cudaError_t _e = (expr);                               \
    if (_e != cudaSuccess) { mxb_set_cuda_error(_e); return MXB_E_CUDA; } \
  } while (0)

#define MXB_LAUNCH_CHECK()                                 \
  do {                                                     \
    mxb_count_launch();                                    \
    cudaError_t _e = cudaGetLastError();                   \
    if (_e != cudaSuccess) { mxb_set_cuda_error(_e); return MXB_E_CUDA; } \
  } while (0)

void mxb_set_cuda_error(cudaError_t e);
void mxb_count_launch();

namespace mxb {

constexpr int kSMs = 148;

__host__ __device__ inline int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

// NaN-propagating max of |v| (torch.amax propagates NaN).
__device__ __forceinline__ float nan_max(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ float nan_min(float a, float b) {
  float r;
  asm("min.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ float amax_step(float acc, float v) { return nan_max(acc, fabsf(v)); }

// Sorted float4 grid (16 entries, -0 before +0) and its 15 bucket
// boundaries fl((g[i]+g[i+1])*0.5), as bit patterns.  Values are the
// normalised E2M1 magnitudes {0,.5,1,1.5,2,3,4,6}/6 and their negatives.
__device__ __constant__ static const uint32_t kF4Grid[16] = {
    0xbf800000u, 0xbf2aaaabu, 0xbf000000u, 0xbeaaaaabu, 0xbe800000u, 0xbe2aaaabu,
    0xbdaaaaabu, 0x80000000u, 0x00000000u, 0x3daaaaabu, 0x3e2aaaabu, 0x3e800000u,
    0x3eaaaaabu, 0x3f000000u, 0x3f2aaaabu, 0x3f800000u};

// Grid value of a code without a memory lookup (lanes holding different
// codes would serialise on the constant cache): index i < 8 is -mag[7 - i],
// i >= 8 is +mag[i - 8], mag = {0, 1/12, 1/6, 1/4, 1/3, 1/2, 2/3, 1} as the
// fp32 bit patterns of kF4Grid; a three-level select picks the magnitude.
__device__ __forceinline__ float f4_grid(int idx) {
  const int i = idx & 15;
  const int j = i ^ (7 + (i >> 3));  // 7 - i below 8, i - 8 from 8
  const uint32_t m01 = (j & 1) ? 0x3daaaaabu : 0x00000000u;  // 1/12 | 0
  const uint32_t m23 = (j & 1) ? 0x3e800000u : 0x3e2aaaabu;  // 1/4 | 1/6
  const uint32_t m45 = (j & 1) ? 0x3f000000u : 0x3eaaaaabu;  // 1/2 | 1/3
  const uint32_t m67 = (j & 1) ? 0x3f800000u : 0x3f2aaaabu;  // 1 | 2/3
  const uint32_t lo = (j & 2) ? m23 : m01, hi = (j & 2) ? m67 : m45;
  const uint32_t mag = (j & 4) ? hi : lo;
  return __uint_as_float(mag | ((i < 8) ? 0x80000000u : 0u));
}

// bucketize(v, mids, right=False) == number of boundaries strictly below v.
// The 15 boundaries are symmetric: -p6..-p0, 0, p0..p6 with p = 1/24, 1/8,
// 5/24, 7/24, 5/12, 7/12, 5/6 (each the fp32 midpoint of adjacent grid
// values).  For v > 0 the count is 8 + #(p < v); for v <= 0 (and -0) it is
// 7 - #(p <= |v|), and p <= a <=> p < nextup(a) for finite a >= 0.  The
// count over the seven p is a three-step branchless binary search.  NaN ->
// 15, as torch.bucketize places NaN last.
__device__ __forceinline__ int f4_bucket(float v) {
  const float p0 = __uint_as_float(0x3d2aaaabu), p1 = 0.125f,
              p2 = __uint_as_float(0x3e555556u), p3 = __uint_as_float(0x3e955556u),
              p4 = __uint_as_float(0x3ed55556u), p5 = __uint_as_float(0x3f155556u),
              p6 = __uint_as_float(0x3f555556u);
  const bool neg = (__float_as_uint(v) >> 31) != 0u;
  const float a = fminf(fabsf(v), 2.0f);  // every p < 2; NaN handled below
  const float x = neg ? __uint_as_float(__float_as_uint(a) + 1u) : a;
  int c = (p3 < x) ? 4 : 0;
  c += (((c & 4) ? p5 : p1) < x) ? 2 : 0;
  const float pl = (c & 4) ? ((c & 2) ? p6 : p4) : ((c & 2) ? p2 : p0);
  c += (pl < x) ? 1 : 0;
  const int i = neg ? 7 - c : 8 + c - (a == 0.0f ? 1 : 0);
  return v == v ? i : 15;
}

// Table form of f4_bucket, for kernels that hold the table in shared memory
// (80 words, f4_tbl_entry(i) for i < 80).  The boundaries 0 < p0 .. p6 are
// compared as bit patterns: t = bits(|v|) + (v < 0) turns the negative side's
// p <= |v| into p < t, as above.  The table has one entry per 1/16 binade
// (t >> 19) from 2^-5 to 2: the number of boundaries below the cell and the
// low 19 bits of the boundary inside it (0x7FFFF if none; no cell holds
// two), so the count is one shared-memory load and one compare instead of
// the three-step search.  Cells below 2^-5 hold only the boundary 0 (t > 0),
// cells from 2 up (NaN included) all eight.  Checked equal to f4_bucket for
// all 2^32 inputs.
__device__ __forceinline__ uint32_t f4_tbl_entry(int i) {
  const uint32_t P[8] = {0u, 0x3d2aaaabu, 0x3e000000u, 0x3e555556u,
                         0x3e955556u, 0x3ed55556u, 0x3f155556u, 0x3f555556u};
  const uint32_t key = 0x7A0u + (uint32_t)i, start = key << 19;
  uint32_t c0 = 0, low = 0x7FFFFu;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    if (P[j] < start) ++c0;
    else if ((P[j] >> 19) == key) low = P[j] & 0x7FFFFu;
  }
  return (c0 << 24) | low;
}

__device__ __forceinline__ int f4_bucket_tbl(float v, const uint32_t* __restrict__ tbl) {
  const uint32_t ng = v < 0.0f ? 1u : 0u;  // NaN counts as positive: index 15
  const uint32_t t = (__float_as_uint(v) & 0x7FFFFFFFu) + ng;
  const int key = min(max((int)(t >> 19), 0x7A0), 0x7EF) - 0x7A0;
  const uint32_t e = tbl[key];
  const int c = (int)(e >> 24) + ((t & 0x7FFFFu) > (e & 0x7FFFFu) ? 1 : 0) - (t == 0u ? 1 : 0);
  return ng ? 8 - c : 7 + c;
}

// Sign-extend the low `bits` bits of v.
__device__ __forceinline__ int sext(uint32_t v, int bits) {
  return (int)(v << (32 - bits)) >> (32 - bits);
}

// Dequantized value of one code (mxtorch.py:1530-1576 per element).
template <int BITS, int KIND>
__device__ __forceinline__ float dequant_code(uint32_t raw, float scale) {
  if (KIND == MXB_KIND_FLOAT) {
    return __fmul_rn(f4_grid((int)(raw & 15u)), scale);
  } else if (BITS == 1) {
    return (raw & 1u) ? -scale : scale;
  } else {
    return __fmul_rn((float)sext(raw, BITS), scale);
  }
}

// ── packed fp32 pairs (add/sub/mul/fma .f32x2, sm_100a): each lane is
// rounded exactly as the scalar .rn instruction would round it.  ptxas may
// fuse a packed mul followed by a packed add, so code that must round the
// product separately keeps its add scalar.
__device__ __forceinline__ uint64_t pack2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ float2 unpack2(uint64_t v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}
__device__ __forceinline__ uint64_t fsub2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t fmul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}

// 32 bits of int4 / int8 codes -> 16/BITS exact float pairs (columns 2p,
// 2p+1): the offset-binary code u (sign bit flipped) placed under exponent
// byte 0x4B reads as 2^23 + u, and one packed subtract removes the offset.
template <int BITS>
__device__ __forceinline__ void decode_word2(uint32_t w, uint64_t* out) {
  if constexpr (BITS == 4) {
    const uint32_t v = w ^ 0x88888888u;  // two's complement -> offset binary (code + 8)
    const uint32_t lo = v & 0x0F0F0F0Fu, hi = (v >> 4) & 0x0F0F0F0Fu;
    const uint64_t bias = pack2(8388616.0f, 8388616.0f);  // 2^23 + 8
#pragma unroll
    for (int k = 0; k < 4; ++k)
      out[k] = fsub2(pack2(__int_as_float(__byte_perm(lo, 0x4B000000u, 0x7440 + k)),
                           __int_as_float(__byte_perm(hi, 0x4B000000u, 0x7440 + k))),
                     bias);
  } else {  // BITS == 8
    const uint32_t v = w ^ 0x80808080u;  // code + 128
    const uint64_t bias = pack2(8388736.0f, 8388736.0f);  // 2^23 + 128
#pragma unroll
    for (int k = 0; k < 2; ++k)
      out[k] = fsub2(pack2(__int_as_float(__byte_perm(v, 0x4B000000u, 0x7440 + 2 * k)),
                           __int_as_float(__byte_perm(v, 0x4B000000u, 0x7441 + 2 * k))),
                     bias);
  }
}

__device__ __forceinline__ float load_as_f32(const float* p, int64_t i) { return __ldg(p + i); }
__device__ __forceinline__ float load_as_f32(const __nv_bfloat16* p, int64_t i) {
  return __bfloat162float(p[i]);
}

}  // namespace mxb
