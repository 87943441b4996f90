// Quantize / pack, dequantize and the randomized Hadamard transform.
//
// All three are HBM-bound byte work.  The vectorised kernels give each
// thread 8 consecutive elements (two 16-byte loads of fp32, one of bf16);
// `block / 8` adjacent lanes own one scale block and reduce its absmax with
// warp shuffles, then each thread writes its 8 packed codes with one store.
// Generic kernels cover the remaining shapes (odd block sizes, unaligned
// pointers).  Rounding follows the reference's fp32 operation order exactly
// (mxtorch.py:1426-1528): reciprocal-then-multiply for the integer scale,
// true division for float4 and for the matmul requantization, round half to
// even.  Built without fast-math so every `__f*_rn` is one IEEE rounding.
#include "mxb_common.cuh"
#include "mxb_internal.h"
#include "wht_regs.cuh"

#include <math.h>
#include <stdint.h>
#include <string.h>

#include <atomic>

using namespace mxb;

namespace {

// Quantizer flavours.
enum QMode { Q_INT_RECIP = 0, Q_INT_DIV = 1, Q_FLOAT4 = 2 };

// Per-block factor: returns scale (stored) and `mul` (what codes use).
template <int BITS, int MODE>
__device__ __forceinline__ void block_factor(float amax, float& scale, float& mul) {
  float a = amax < 1e-12f ? 1e-12f : amax;  // clamp(min=1e-12), NaN kept
  if (MODE == Q_FLOAT4 || (MODE == Q_INT_RECIP && BITS == 1)) {
    scale = a;
    mul = a;
  } else if (MODE == Q_INT_RECIP) {
    const float max_int = (float)((1 << (BITS - 1)) - 1);
    float si = __fmul_rn(__frcp_rn(a), max_int);  // max_int / a  (torch __rdiv__)
    scale = __frcp_rn(si);                        // scale_inv.reciprocal()
    mul = si;
  } else {  // Q_INT_DIV: requantization of the matmul output
    const float max_out = (float)((1 << (BITS - 1)) - 1);
    scale = __fdiv_rn(a, max_out);
    mul = scale;
  }
}

// NAN_SELECT false: the caller has checked that the block's multiplier (or
// divisor) is finite and positive, so no quotient is NaN (see quant8_store).
template <int BITS, int MODE, bool NAN_SELECT = true>
__device__ __forceinline__ uint32_t code_of(float v, float mul) {
  if (MODE == Q_FLOAT4) {
    return (uint32_t)f4_bucket(__fdiv_rn(v, mul));
  } else if (MODE == Q_INT_RECIP && BITS == 1) {
    return (v >= 0.0f) ? 0u : 1u;  // where(x >= 0, 0, -1); NaN -> -1
  } else {
    const float m = (float)((1 << (BITS - 1)) - 1);
    float q = (MODE == Q_INT_RECIP) ? __fmul_rn(v, mul) : __fdiv_rn(v, mul);
    // The reference clamps q to [-m, m] before rounding; here that clamp
    // never changes a code, so it is left out.  Every |x| of a block is at
    // most a = max(amax, 1e-12), and mul = fl(fl(1/a) * m) (or the divisor
    // fl(a / m)), so |q| <= m (1 + 2^-24)^3 < m + 0.5, which rounds to m; a
    // block whose amax is inf or NaN makes q 0 or NaN either way.
    (void)m;
    // Round half to even by adding 1.5 * 2^23 (|q| <= 32767 < 2^22): the sum's
    // low mantissa bits are the two's-complement code.  NaN stores code 0, as
    // the reference's NaN -> int conversion does.
    const uint32_t c = __float_as_uint(__fadd_rn(q, 12582912.0f)) & ((1u << BITS) - 1u);
    return (!NAN_SELECT || q == q) ? c : 0u;
  }
}

// Quantize E (8 or 16) consecutive values owned by this lane; `L` lanes form
// a block.  Writes the packed codes of these elements at byte offset
// (e0 * BITS / 8).  With 16 per lane the block's absmax shuffles and scale
// computation are shared by twice as many elements.
// f4t: the float4 bucket table in shared memory (f4_bucket_tbl), or nullptr.
template <int BITS, int MODE, int E = 8>
__device__ __forceinline__ void quant8_store(const float (&v)[E], bool valid, int L,
                                             int64_t e0, uint8_t* __restrict__ packed,
                                             float* __restrict__ scales, int64_t blk,
                                             const uint32_t* f4t = nullptr) {
  float a = 0.0f;
#pragma unroll
  for (int i = 0; i < E; ++i) a = amax_step(a, v[i]);
  for (int o = L >> 1; o > 0; o >>= 1) a = nan_max(a, __shfl_xor_sync(0xffffffffu, a, o));
  if (!valid) return;
  float scale, mul;
  block_factor<BITS, MODE>(a, scale, mul);
  if ((threadIdx.x & (L - 1)) == 0) scales[blk] = scale;
  uint32_t cc[E];
#pragma unroll
  for (int i = 0; i < E; ++i)
    cc[i] = (MODE == Q_FLOAT4 && f4t != nullptr)
                ? (uint32_t)f4_bucket_tbl(__fdiv_rn(v[i], mul), f4t)
                : code_of<BITS, MODE, MODE == Q_FLOAT4 || BITS == 1>(v[i], mul);
  if (MODE != Q_FLOAT4 && BITS != 1 && !(mul > 0.0f && mul <= 3.4028235e38f)) {
    // A NaN in the block makes amax and mul NaN, an inf makes the multiplier
    // 0 (the divisor inf): every quotient is then 0 or NaN, and every code 0.
    // A finite positive mul means every x of the block is finite, so no
    // quotient is NaN and the per-element NaN test above is not needed.
#pragma unroll
    for (int i = 0; i < E; ++i) cc[i] = 0u;
  }
#pragma unroll
  for (int h = 0; h < E / 8; ++h) {
  const uint32_t* c = cc + 8 * h;
  uint8_t* p = packed + ((e0 + 8 * h) * BITS) / 8;
  if (BITS == 8) {
    uint2 w;
    w.x = c[0] | (c[1] << 8) | (c[2] << 16) | (c[3] << 24);
    w.y = c[4] | (c[5] << 8) | (c[6] << 16) | (c[7] << 24);
    *reinterpret_cast<uint2*>(p) = w;
  } else if (BITS == 16) {
    uint4 w;
    w.x = c[0] | (c[1] << 16);
    w.y = c[2] | (c[3] << 16);
    w.z = c[4] | (c[5] << 16);
    w.w = c[6] | (c[7] << 16);
    *reinterpret_cast<uint4*>(p) = w;
  } else if (BITS == 4) {
    uint32_t w = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) w |= c[i] << (4 * i);
    *reinterpret_cast<uint32_t*>(p) = w;
  } else if (BITS == 2) {
    uint32_t w = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) w |= c[i] << (2 * i);
    *reinterpret_cast<uint16_t*>(p) = (uint16_t)w;
  } else {  // BITS == 1
    uint32_t w = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) w |= c[i] << i;
    *p = (uint8_t)w;
  }
  }
}

template <typename InT>
__device__ __forceinline__ void load8(const InT* __restrict__ x, int64_t e0, int64_t n,
                                      bool vec, float (&v)[8]) {
  if (vec && e0 + 8 <= n) {
    if (sizeof(InT) == 4) {
      const float4* p = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(x) + e0);
      float4 a = __ldcs(p), b = __ldcs(p + 1);
      v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
      v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    } else {
      uint4 r = __ldcs(reinterpret_cast<const uint4*>(
          reinterpret_cast<const __nv_bfloat16*>(x) + e0));
      uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        v[2 * i] = __uint_as_float(w[i] << 16);
        v[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = (e0 + i < n) ? load_as_f32(x, e0 + i) : 0.0f;
  }
}

// Vectorised quantize: block in {8,16,32,64,128,256}; E elements per lane
// (16 needs block % 16 == 0).
template <typename InT, int BITS, int MODE, int E = 8>
__global__ void __launch_bounds__(256) quant_vec_kernel(const InT* __restrict__ x, int64_t n,
                                                        int block, int64_t nb, bool vec,
                                                        uint8_t* __restrict__ packed,
                                                        float* __restrict__ scales) {
  const int L = block / E;
  const int64_t groups = nb * (int64_t)L;  // threads with work
  const int lane = threadIdx.x & 31;
  const int64_t warp0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  __shared__ uint32_t f4s[MODE == Q_FLOAT4 ? 80 : 1];
  const uint32_t* f4t = nullptr;
  if constexpr (MODE == Q_FLOAT4) {
    for (int i = threadIdx.x; i < 80; i += blockDim.x) f4s[i] = f4_tbl_entry(i);
    __syncthreads();
    f4t = f4s;
  }
#ifndef MXB_Q_BF16_PREFETCH
#define MXB_Q_BF16_PREFETCH 1
#endif
  if constexpr (sizeof(InT) == 2 && MXB_Q_BF16_PREFETCH) {
    // bf16: a lane's E inputs are only 2E bytes, so the next iteration's
    // words are loaded before this one is quantized (twice the bytes in
    // flight per lane).  Lanes whose group is not whole take load8.
    const uint4* xv = reinterpret_cast<const uint4*>(x);
    uint4 raw[E / 8];
    auto fetch = [&](int64_t tt) {
      if (vec && tt * E + E <= n) {
#pragma unroll
        for (int h = 0; h < E / 8; ++h) raw[h] = __ldcs(xv + (tt * E) / 8 + h);
      }
    };
    fetch(warp0 * 32 + lane);
    for (int64_t w = warp0; w * 32 < groups; w += nwarps) {
      const int64_t t = w * 32 + lane;
      const bool valid = t < groups;
      float v[E];
      if (vec && t * E + E <= n) {
#pragma unroll
        for (int h = 0; h < E / 8; ++h) {
          const uint32_t wd[4] = {raw[h].x, raw[h].y, raw[h].z, raw[h].w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            v[8 * h + 2 * i] = __uint_as_float(wd[i] << 16);
            v[8 * h + 2 * i + 1] = __uint_as_float(wd[i] & 0xffff0000u);
          }
        }
      } else {
#pragma unroll
        for (int h = 0; h < E / 8; ++h)
          load8<InT>(x, t * E + 8 * h, valid ? n : 0, vec,
                     *reinterpret_cast<float(*)[8]>(v + 8 * h));
      }
      fetch(t + nwarps * 32);
      quant8_store<BITS, MODE, E>(v, valid, L, t * E, packed, scales, t / L, f4t);
    }
  } else {
    for (int64_t w = warp0; w * 32 < groups; w += nwarps) {
      const int64_t t = w * 32 + lane;
      const bool valid = t < groups;
      float v[E];
#pragma unroll
      for (int h = 0; h < E / 8; ++h)
        load8<InT>(x, t * E + 8 * h, valid ? n : 0, vec,
                   *reinterpret_cast<float(*)[8]>(v + 8 * h));
      quant8_store<BITS, MODE, E>(v, valid, L, t * E, packed, scales, t / L, f4t);
    }
  }
}

// Generic pass 1: one warp per block -> scale and code multiplier.
template <typename InT, int BITS, int MODE>
__global__ void __launch_bounds__(256) quant_scales_kernel(const InT* __restrict__ x, int64_t n,
                                                           int block, int64_t nb,
                                                           float* __restrict__ scales,
                                                           float* __restrict__ muls) {
  const int lane = threadIdx.x & 31;
  int64_t b = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (; b < nb; b += nw) {
    float a = 0.0f;
    const int64_t e0 = b * block;
    for (int i = lane; i < block; i += 32) {
      int64_t e = e0 + i;
      if (e < n) a = amax_step(a, load_as_f32(x, e));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) a = nan_max(a, __shfl_xor_sync(0xffffffffu, a, o));
    if (lane == 0) {
      float s, m;
      block_factor<BITS, MODE>(a, s, m);
      scales[b] = s;
      muls[b] = m;
    }
  }
}

// Generic pass 2: one thread per packed storage word (8 bits, or 32 for 16-bit codes).
template <typename InT, int BITS, int MODE>
__global__ void __launch_bounds__(256) quant_pack_kernel(const InT* __restrict__ x, int64_t n,
                                                         int block, int64_t ncodes,
                                                         int64_t nwords,
                                                         const float* __restrict__ muls,
                                                         uint8_t* __restrict__ packed) {
  constexpr int WBITS = BITS == 16 ? 32 : 8;
  constexpr int PER = WBITS / BITS;
  for (int64_t wi = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; wi < nwords;
       wi += (int64_t)gridDim.x * blockDim.x) {
    uint32_t word = 0;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      int64_t e = wi * PER + i;
      if (e >= ncodes) break;  // storage padding beyond the last block: code 0
      float v = e < n ? load_as_f32(x, e) : 0.0f;
      word |= code_of<BITS, MODE>(v, muls[e / block]) << (i * BITS);
    }
    if (BITS == 16)
      reinterpret_cast<uint32_t*>(packed)[wi] = word;
    else
      packed[wi] = (uint8_t)word;
  }
}

// ── dequantize ───────────────────────────────────────────────────────────────
template <int BITS>
__device__ __forceinline__ uint32_t raw_code(const uint8_t* __restrict__ packed, int64_t e) {
  if constexpr (BITS == 16) {
    uint32_t w = __ldg(reinterpret_cast<const uint32_t*>(packed) + (e >> 1));
    return (w >> ((e & 1) * 16)) & 0xffffu;
  }
  constexpr int PER = BITS >= 8 ? 1 : 8 / BITS;
  uint32_t b = __ldg(packed + e / PER);
  return (b >> ((e % PER) * BITS)) & ((1u << BITS) - 1u);
}

// 8 elements per lane and group (two float4 stores per lane), two groups
// per iteration: cheaper per element where the decode itself is the cost.
template <int BITS, int KIND>
__device__ __forceinline__ void load_codes8(const uint8_t* __restrict__ packed, int64_t e0,
                                            uint32_t (&w)[4]) {
  const uint8_t* p = packed + (e0 * BITS) / 8;
  if (BITS == 16) {
    const uint4 v = __ldcs(reinterpret_cast<const uint4*>(p));
    w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
  } else if (BITS == 8) {
    const uint2 v = __ldcs(reinterpret_cast<const uint2*>(p));
    w[0] = v.x; w[1] = v.y;
  } else if (BITS == 4) {
    w[0] = __ldcs(reinterpret_cast<const uint32_t*>(p));
  } else if (BITS == 2) {
    w[0] = __ldcs(reinterpret_cast<const uint16_t*>(p));
  } else {
    w[0] = *p;
  }
}

// tbl: the float4 grid in shared memory (float4 only; nullptr otherwise)
template <int BITS, int KIND>
__device__ __forceinline__ void dequant8_store(const uint32_t (&w)[4], float s, int64_t e0,
                                               int64_t n, float* __restrict__ out,
                                               const float* tbl = nullptr) {
  uint32_t c[8];
  if (BITS == 8) {
#pragma unroll
    for (int i = 0; i < 4; ++i) { c[i] = (w[0] >> (8 * i)) & 0xff; c[i + 4] = (w[1] >> (8 * i)) & 0xff; }
  } else if (BITS == 16) {
#pragma unroll
    for (int i = 0; i < 4; ++i) { c[2 * i] = w[i] & 0xffff; c[2 * i + 1] = w[i] >> 16; }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) c[i] = (w[0] >> (BITS * i)) & ((1u << BITS) - 1u);
  }
  float r[8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
    r[i] = KIND == MXB_KIND_FLOAT ? __fmul_rn(tbl[c[i] & 15u], s) : dequant_code<BITS, KIND>(c[i], s);
  if (e0 + 8 <= n) {
    float4* o = reinterpret_cast<float4*>(out + e0);
    __stcs(o, make_float4(r[0], r[1], r[2], r[3]));
    __stcs(o + 1, make_float4(r[4], r[5], r[6], r[7]));
  } else {
    for (int i = 0; i < 8; ++i)
      if (e0 + i < n) out[e0 + i] = r[i];
  }
}

template <int BITS, int KIND>
__global__ void __launch_bounds__(256) dequant_vec8_kernel(const uint8_t* __restrict__ packed,
                                                           const float* __restrict__ scales,
                                                           int64_t n, int block,
                                                           float* __restrict__ out) {
  // float4: the 16 grid values in shared memory, one bank each, so lanes
  // reading different codes do not conflict (one load per value instead of
  // a select chain)
  __shared__ float tbl[16];
  if (KIND == MXB_KIND_FLOAT) {
    if (threadIdx.x < 16) tbl[threadIdx.x] = f4_grid((int)threadIdx.x);
    __syncthreads();
  }
  const int64_t ngroups = (n + 7) / 8;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < ngroups; t += 2 * stride) {
    const int64_t t2 = t + stride;
    const bool two = t2 < ngroups;
    uint32_t wa[4] = {0u, 0u, 0u, 0u}, wb[4] = {0u, 0u, 0u, 0u};
    load_codes8<BITS, KIND>(packed, t * 8, wa);
    const float sa = __ldg(scales + (t * 8) / block);
    float sb = 0.0f;
    if (two) {
      load_codes8<BITS, KIND>(packed, t2 * 8, wb);
      sb = __ldg(scales + (t2 * 8) / block);
    }
    dequant8_store<BITS, KIND>(wa, sa, t * 8, n, out, tbl);
    if (two) dequant8_store<BITS, KIND>(wb, sb, t2 * 8, n, out, tbl);
  }
}

// Codes of 4 consecutive elements starting at e0 (e0 % 4 == 0), low bits first.
template <int BITS>
__device__ __forceinline__ uint64_t load_codes4(const uint8_t* __restrict__ packed, int64_t e0) {
  if (BITS == 16) {
    const uint2 v = __ldcs(reinterpret_cast<const uint2*>(packed + e0 * 2));
    return (uint64_t)v.x | ((uint64_t)v.y << 32);
  } else if (BITS == 8) {
    return __ldcs(reinterpret_cast<const uint32_t*>(packed + e0));
  } else if (BITS == 4) {
    return __ldcs(reinterpret_cast<const uint16_t*>(packed + e0 / 2));
  } else if (BITS == 2) {
    return __ldcs(packed + e0 / 4);
  } else {
    return (uint64_t)(__ldcs(packed + e0 / 8) >> (e0 & 4));
  }
}

// Fused activations after dequantize.  ReLU keeps NaN (torch's CPU relu
// propagates it); SiLU(g) = g / (1 + exp(-g)).
enum DqAct { ACT_NONE = 0, ACT_RELU = 1 };
__device__ __forceinline__ float relu_keep_nan(float v) {
  return v > 0.0f ? v : (v != v ? v : 0.0f);
}
__device__ __forceinline__ float silu(float g) { return __fdiv_rn(g, __fadd_rn(1.0f, expf(-g))); }

template <int BITS, int KIND>
__device__ __forceinline__ void dequant4(uint64_t w, float s, const float* tbl, float (&r)[4]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t raw = (uint32_t)(w >> (BITS * i)) & (uint32_t)((1ull << BITS) - 1u);
    r[i] = KIND == MXB_KIND_FLOAT ? __fmul_rn(tbl[raw & 15u], s) : dequant_code<BITS, KIND>(raw, s);
  }
}

template <int BITS, int KIND, int ACT = ACT_NONE>
__device__ __forceinline__ void dequant4_store(uint64_t w, float s, int64_t e0, int64_t n,
                                               float* __restrict__ out, const float* tbl) {
  float r[4];
  dequant4<BITS, KIND>(w, s, tbl, r);
  if (ACT == ACT_RELU) {
#pragma unroll
    for (int i = 0; i < 4; ++i) r[i] = relu_keep_nan(r[i]);
  }
  if (e0 + 4 <= n) {
    __stcs(reinterpret_cast<float4*>(out + e0), make_float4(r[0], r[1], r[2], r[3]));
  } else {
    for (int i = 0; i < 4; ++i)
      if (e0 + i < n) out[e0 + i] = r[i];
  }
}

// 4 elements per lane and group, so each warp store covers 512 contiguous
// bytes; four groups per iteration, all loads issued before any is used.
template <int BITS, int KIND>
__global__ void __launch_bounds__(256) dequant_vec_kernel(const uint8_t* __restrict__ packed,
                                                          const float* __restrict__ scales,
                                                          int64_t n, int block,
                                                          float* __restrict__ out) {
  constexpr int U = 4;
  __shared__ float tbl[16];  // float4 grid (see dequant_vec8_kernel)
  if (KIND == MXB_KIND_FLOAT) {
    if (threadIdx.x < 16) tbl[threadIdx.x] = f4_grid((int)threadIdx.x);
    __syncthreads();
  }
  const int64_t ngroups = (n + 3) / 4;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < ngroups; t += U * stride) {
    uint64_t w[U];
    float sc[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t g = t + u * stride;
      w[u] = 0;
      sc[u] = 0.0f;
      if (g < ngroups) {
        w[u] = load_codes4<BITS>(packed, g * 4);
        sc[u] = __ldg(scales + (g * 4) / block);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t g = t + u * stride;
      if (g < ngroups) dequant4_store<BITS, KIND>(w[u], sc[u], g * 4, n, out, tbl);
    }
  }
}

// Warp-chunk dequantize (BITS <= 8): one warp per 1024-element chunk,
// 32*BITS packed words.  Lane l reads words l, l+32, ... (BITS coalesced
// 128-byte warp loads), then the warp writes 8 float4 rows of 128 elements.
// Row j's 4 codes for lane l start at chunk bit 4*BITS*(32j + l), i.e. in
// word j*4*BITS + l*BITS/8: register (j*4*BITS)/32 of lane (that word) % 32,
// a register index fixed per row, so one shuffle delivers it.  Every store
// instruction covers 512 contiguous bytes.  Words past the end of the packed
// buffer are read byte by byte.
template <int BITS, int KIND, int ACT = ACT_NONE>
__global__ void __launch_bounds__(256) dequant_warp_kernel(const uint8_t* __restrict__ packed,
                                                           const float* __restrict__ scales,
                                                           int64_t n, int block,
                                                           float* __restrict__ out) {
  static_assert(BITS <= 8, "warp-chunk dequantize covers codes up to 8 bits");
  __shared__ float tbl[16];  // float4 grid (see dequant_vec8_kernel)
  if (KIND == MXB_KIND_FLOAT) {
    if (threadIdx.x < 16) tbl[threadIdx.x] = f4_grid((int)threadIdx.x);
    __syncthreads();
  }
  const int lane = threadIdx.x & 31;
  const int64_t nbytes = (n * BITS + 7) / 8;
  const int64_t nchunks = (n + 1023) / 1024;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t c = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; c < nchunks;
       c += nwarps) {
    uint32_t word[BITS];
#pragma unroll
    for (int k = 0; k < BITS; ++k) {
      const int64_t b0 = ((c * BITS + k) * 32 + lane) * 4;
      word[k] = 0u;
      if (b0 + 4 <= nbytes) {
        word[k] = __ldcs(reinterpret_cast<const uint32_t*>(packed + b0));
      } else {
        for (int i = 0; i < 4; ++i)
          if (b0 + i < nbytes) word[k] |= (uint32_t)packed[b0 + i] << (8 * i);
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      constexpr int kRowWords = 4 * BITS;  // packed words per 128-element row
      const uint32_t src = __shfl_sync(0xffffffffu, word[(j * kRowWords) >> 5],
                                       ((j * kRowWords) & 31) + (lane * BITS) / 8);
      const int64_t e0 = c * 1024 + j * 128 + lane * 4;
      if (e0 < n)
        dequant4_store<BITS, KIND, ACT>(src >> ((lane * 4 * BITS) & 31), __ldg(scales + e0 / block),
                                   e0, n, out, tbl);
    }
  }
}

template <int BITS, int KIND, int ACT = ACT_NONE>
__global__ void __launch_bounds__(256) dequant_generic_kernel(const uint8_t* __restrict__ packed,
                                                              const float* __restrict__ scales,
                                                              int64_t n, int block,
                                                              float* __restrict__ out) {
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n;
       e += (int64_t)gridDim.x * blockDim.x) {
    const float v = dequant_code<BITS, KIND>(raw_code<BITS>(packed, e), __ldg(scales + e / block));
    out[e] = ACT == ACT_RELU ? relu_keep_nan(v) : v;
  }
}

// SiLU(dequant(gate)) * dequant(up) (mxtorch.py:3459-3479, 4077-4109), both
// operands of one dtype, block and length.  Same warp-chunk layout as
// dequant_warp_kernel, over two packed streams.
template <int BITS, int KIND>
__global__ void __launch_bounds__(256) silu_mul_warp_kernel(
    const uint8_t* __restrict__ gp, const float* __restrict__ gs, const uint8_t* __restrict__ up,
    const float* __restrict__ us, int64_t n, int block, float* __restrict__ out) {
  static_assert(BITS <= 8, "warp-chunk kernels cover codes up to 8 bits");
  __shared__ float tbl[16];
  if (KIND == MXB_KIND_FLOAT) {
    if (threadIdx.x < 16) tbl[threadIdx.x] = f4_grid((int)threadIdx.x);
    __syncthreads();
  }
  const int lane = threadIdx.x & 31;
  const int64_t nbytes = (n * BITS + 7) / 8;
  const int64_t nchunks = (n + 1023) / 1024;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t c = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; c < nchunks;
       c += nwarps) {
    uint32_t wg[BITS], wu[BITS];
#pragma unroll
    for (int k = 0; k < BITS; ++k) {
      const int64_t b0 = ((c * BITS + k) * 32 + lane) * 4;
      wg[k] = wu[k] = 0u;
      if (b0 + 4 <= nbytes) {
        wg[k] = __ldcs(reinterpret_cast<const uint32_t*>(gp + b0));
        wu[k] = __ldcs(reinterpret_cast<const uint32_t*>(up + b0));
      } else {
        for (int i = 0; i < 4; ++i)
          if (b0 + i < nbytes) {
            wg[k] |= (uint32_t)gp[b0 + i] << (8 * i);
            wu[k] |= (uint32_t)up[b0 + i] << (8 * i);
          }
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      constexpr int kRowWords = 4 * BITS;
      const int reg = (j * kRowWords) >> 5;
      const int srcl = ((j * kRowWords) & 31) + (lane * BITS) / 8;
      const int sh = (lane * 4 * BITS) & 31;
      const uint32_t g = __shfl_sync(0xffffffffu, wg[reg], srcl) >> sh;
      const uint32_t u = __shfl_sync(0xffffffffu, wu[reg], srcl) >> sh;
      const int64_t e0 = c * 1024 + j * 128 + lane * 4;
      if (e0 < n) {
        float rg[4], ru[4];
        dequant4<BITS, KIND>(g, __ldg(gs + e0 / block), tbl, rg);
        dequant4<BITS, KIND>(u, __ldg(us + e0 / block), tbl, ru);
        float r[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) r[i] = __fmul_rn(silu(rg[i]), ru[i]);
        if (e0 + 4 <= n) {
          __stcs(reinterpret_cast<float4*>(out + e0), make_float4(r[0], r[1], r[2], r[3]));
        } else {
          for (int i = 0; i < 4; ++i)
            if (e0 + i < n) out[e0 + i] = r[i];
        }
      }
    }
  }
}

template <int BITS, int KIND>
__global__ void __launch_bounds__(256) silu_mul_generic_kernel(
    const uint8_t* __restrict__ gp, const float* __restrict__ gs, const uint8_t* __restrict__ up,
    const float* __restrict__ us, int64_t n, int block, float* __restrict__ out) {
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n;
       e += (int64_t)gridDim.x * blockDim.x) {
    const float g = dequant_code<BITS, KIND>(raw_code<BITS>(gp, e), __ldg(gs + e / block));
    const float u = dequant_code<BITS, KIND>(raw_code<BITS>(up, e), __ldg(us + e / block));
    out[e] = __fmul_rn(silu(g), u);
  }
}

// ── Walsh–Hadamard transform of one row held in shared memory ────────────────
// Stage order is the reference's (mxtorch.py:2811-2832): stride n/2 first,
// down to 1, each pair (e, o) -> (e + o, e - o).  Strides >= 32 run as
// radix-2^R passes in registers; strides < 32 with warp shuffles.
template <int R>
__device__ __forceinline__ void wht_pass(float* s, int n, int lo) {
  constexpr int RR = 1 << R;
  const int nbase = n >> R;
  const int hi = lo + R;
  for (int b = threadIdx.x; b < nbase; b += blockDim.x) {
    const int base = (b & ((1 << lo) - 1)) | ((b >> lo) << hi);
    float v[RR];
#pragma unroll
    for (int j = 0; j < RR; ++j) v[j] = s[base + (j << lo)];
#pragma unroll
    for (int q = R - 1; q >= 0; --q) {
#pragma unroll
      for (int j = 0; j < RR; ++j) {
        if (!(j & (1 << q))) {
          float e = v[j], o = v[j + (1 << q)];
          v[j] = __fadd_rn(e, o);
          v[j + (1 << q)] = __fsub_rn(e, o);
        }
      }
    }
#pragma unroll
    for (int j = 0; j < RR; ++j) s[base + (j << lo)] = v[j];
  }
}

// In-warp stages for strides min(n,32)/2 .. 1 on value v at index i (lane = i & 31).
__device__ __forceinline__ float wht_low(float v, int n) {
  const int lane = threadIdx.x & 31;
  const int top = n < 32 ? n : 32;
  for (int h = top >> 1; h > 0; h >>= 1) {
    float p = __shfl_xor_sync(0xffffffffu, v, h);
    v = (lane & h) ? __fsub_rn(p, v) : __fadd_rn(v, p);
  }
  return v;
}

// Full transform (without the 1/sqrt(n)); leaves the result in s.
__device__ void wht_row(float* s, int n) {
  int L = 31 - __clz(n);
  int hi = L;
  while (hi > 5) {
    int r = hi - 5 < 4 ? hi - 5 : 4;
    int lo = hi - r;
    __syncthreads();
    switch (r) {
      case 4: wht_pass<4>(s, n, lo); break;
      case 3: wht_pass<3>(s, n, lo); break;
      case 2: wht_pass<2>(s, n, lo); break;
      default: wht_pass<1>(s, n, lo); break;
    }
    hi = lo;
  }
  __syncthreads();
  const int span = n < 32 ? 32 : n;
  for (int i0 = threadIdx.x & ~31; i0 < span; i0 += blockDim.x) {
    int i = i0 + (threadIdx.x & 31);
    float v = (i < n) ? s[i] : 0.0f;
    v = wht_low(v, n);
    if (i < n) s[i] = v;
  }
  __syncthreads();
}

// Load one row: s[i] = x[i] * sign[i] (rotate) or x[i] (unrotate) for i < d, 0 above.
template <typename InT>
__device__ __forceinline__ void load_row(float* s, const InT* __restrict__ xr, int d, int n,
                                         const float* __restrict__ signs, bool mul_signs) {
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    float v = 0.0f;
    if (i < d) {
      v = load_as_f32(xr, i);
      if (mul_signs) v = __fmul_rn(v, __ldg(signs + i));
    }
    s[i] = v;
  }
}

// Rotate each row, then (fuse_quant) quantize it in place, or write the
// rotated fp32 row to `rot_out`.
template <typename InT, int BITS, int MODE>
__global__ void __launch_bounds__(256) hquant_kernel(const InT* __restrict__ x, int d, int n,
                                                     float sqrtn, const float* __restrict__ signs,
                                                     int block, bool fuse_quant,
                                                     uint8_t* __restrict__ packed,
                                                     float* __restrict__ scales,
                                                     float* __restrict__ rot_out) {
  extern __shared__ __align__(16) float srow[];
  const int64_t r = blockIdx.x;
  load_row<InT>(srow, x + r * d, d, n, signs, true);
  wht_row(srow, n);
  for (int i = threadIdx.x; i < d; i += blockDim.x) srow[i] = __fdiv_rn(srow[i], sqrtn);
  __syncthreads();
  if (!fuse_quant) {
    for (int i = threadIdx.x; i < d; i += blockDim.x) rot_out[r * d + i] = srow[i];
    return;
  }
  // d % block == 0 and block in {8..256}: blocks are row-local.
  const int L = block / 8;
  const int groups = d / 8;
  const int lane = threadIdx.x & 31;
  const int64_t row_e0 = r * (int64_t)d;
  const int64_t row_b0 = row_e0 / block;
  for (int w = (threadIdx.x >> 5) * 32; w < groups; w += blockDim.x) {
    const int t = w + lane;
    const bool valid = t < groups;
    float v[8];
    if (valid) {
      float4 a = *reinterpret_cast<const float4*>(srow + 8 * t);
      float4 b = *reinterpret_cast<const float4*>(srow + 8 * t + 4);
      v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
      v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = 0.0f;
    }
    quant8_store<BITS, MODE>(v, valid, L, row_e0 + 8 * t, packed, scales, row_b0 + t / L);
  }
}

// Dequantize each row's codes, then unrotate.
template <int BITS, int KIND>
__global__ void __launch_bounds__(256) hdequant_kernel(const uint8_t* __restrict__ packed,
                                                       const float* __restrict__ scales,
                                                       int d, int n, float sqrtn,
                                                       const float* __restrict__ signs,
                                                       int block, float* __restrict__ out) {
  extern __shared__ __align__(16) float srow[];
  const int64_t r = blockIdx.x;
  const int64_t e0 = r * (int64_t)d;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    float v = 0.0f;
    if (i < d) {
      int64_t e = e0 + i;
      v = dequant_code<BITS, KIND>(raw_code<BITS>(packed, e), __ldg(scales + e / block));
    }
    srow[i] = v;
  }
  wht_row(srow, n);
  for (int i = threadIdx.x; i < d; i += blockDim.x)
    out[e0 + i] = __fmul_rn(__fdiv_rn(srow[i], sqrtn), __ldg(signs + i));
}

__global__ void __launch_bounds__(256) hrows_kernel(const float* __restrict__ x, int d, int n,
                                                    float sqrtn, const float* __restrict__ signs,
                                                    bool inverse, float* __restrict__ out) {
  extern __shared__ __align__(16) float srow[];
  const int64_t r = blockIdx.x;
  load_row<float>(srow, x + r * d, d, n, signs, !inverse);
  wht_row(srow, n);  // begins and ends with __syncthreads, so in-place is safe
  for (int i = threadIdx.x; i < d; i += blockDim.x) {
    float v = __fdiv_rn(srow[i], sqrtn);
    if (inverse) v = __fmul_rn(v, __ldg(signs + i));
    out[r * d + i] = v;
  }
}

// ── the same three kernels with the row in registers (n = 256 * V) ─────────
// Bit-identical to the shared-memory versions above (same stage order and
// rounding, whtr::div_sqrtn equal to the IEEE quotient where selected); two
// passes through shared memory instead of one per radix pass plus the
// shuffle stages, and the row leaves in runs of consecutive elements.

template <typename InT, int BITS, int MODE, int V>
__global__ void __launch_bounds__(256) hquant_fast_kernel(
    const InT* __restrict__ x, int d, float sqrtn, float rsq, int dmode,
    const float* __restrict__ signs, int block, bool fuse_quant, uint8_t* __restrict__ packed,
    float* __restrict__ scales, float* __restrict__ rot_out) {
  using W = whtr::Row<V>;
  extern __shared__ __align__(16) float srow[];
  const int64_t r = blockIdx.x;
  const InT* xr = x + r * d;
  const int t = threadIdx.x;
  float v[V];
  if (W::kPhaseC && W::kG >= 8 && d % W::kG == 0 && ((uintptr_t)xr & 15) == 0) {
    // the row in runs of kG consecutive elements (16-byte loads), times the
    // signs, then to the phase-A layout through shared memory
#pragma unroll
    for (int q = 0; q < W::kRuns; ++q) {
      const int i0 = W::idx(t, q * W::kG);
#pragma unroll
      for (int c8 = 0; c8 < W::kG / 8; ++c8) {
        float a[8];
        if (i0 < d) {
          load8<InT>(xr, i0 + 8 * c8, d, true, a);
          const float4 s0 = __ldg(reinterpret_cast<const float4*>(signs + i0 + 8 * c8));
          const float4 s1 = __ldg(reinterpret_cast<const float4*>(signs + i0 + 8 * c8) + 1);
          const float sg[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
#pragma unroll
          for (int c = 0; c < 8; ++c) a[c] = __fmul_rn(a[c], sg[c]);
        } else {
#pragma unroll
          for (int c = 0; c < 8; ++c) a[c] = 0.0f;
        }
#pragma unroll
        for (int c = 0; c < 8; ++c) v[q * W::kG + 8 * c8 + c] = a[c];
      }
    }
    if constexpr (W::kPhaseC) W::from_runs(v, srow);
  } else {
#pragma unroll
    for (int j = 0; j < V; ++j) {
      const int i = W::idxA(t, j);
      v[j] = i < d ? __fmul_rn(load_as_f32(xr, i), __ldg(signs + i)) : 0.0f;
    }
  }
  W::transform(v, srow);
#pragma unroll
  for (int j = 0; j < V; ++j) v[j] = whtr::div_sqrtn(v[j], sqrtn, rsq, dmode);
  if (!fuse_quant) {
#pragma unroll
    for (int j = 0; j < V; ++j) {
      const int i = W::idx(t, j);
      if (i < d) rot_out[r * d + i] = v[j];
    }
    return;
  }
  const int64_t row_e0 = r * (int64_t)d;
  constexpr int E = W::kG;  // run length: 8 or 16 consecutive elements
  if constexpr (W::kPhaseC && (E == 8 || E == 16)) {
    if (block % E == 0) {
      // runs of E consecutive elements in consecutive lanes: block / E lanes
      // form a block, exactly the layout quant8_store takes
      const int L = block / E;
#pragma unroll
      for (int q = 0; q < W::kRuns; ++q) {
        const int i0 = W::idx(t, q * E);
        const bool valid = i0 < d;
        quant8_store<BITS, MODE, E>(*reinterpret_cast<float(*)[E]>(v + q * E), valid, L,
                                    row_e0 + i0, packed, scales, (row_e0 + i0) / block);
      }
      return;
    }
  }
  // other run lengths: through shared memory in natural order
#pragma unroll
  for (int j = 0; j < V; ++j) {
    const int i = W::idx(t, j);
    if (i < d) srow[i] = v[j];
  }
  __syncthreads();
  // d % block == 0 and block in {8..256}: blocks are row-local.
  const int L = block / 8;
  const int groups = d / 8;
  const int lane = threadIdx.x & 31;
  const int64_t row_b0 = row_e0 / block;
  for (int w = (threadIdx.x >> 5) * 32; w < groups; w += blockDim.x) {
    const int tt = w + lane;
    const bool valid = tt < groups;
    float q[8];
    if (valid) {
      float4 a = *reinterpret_cast<const float4*>(srow + 8 * tt);
      float4 b = *reinterpret_cast<const float4*>(srow + 8 * tt + 4);
      q[0] = a.x; q[1] = a.y; q[2] = a.z; q[3] = a.w;
      q[4] = b.x; q[5] = b.y; q[6] = b.z; q[7] = b.w;
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) q[i] = 0.0f;
    }
    quant8_store<BITS, MODE>(q, valid, L, row_e0 + 8 * tt, packed, scales, row_b0 + tt / L);
  }
}

// Final stage of the row kernels: out[i] = div(v, sqrt n) (times signs[i]
// when `sgn`), in runs of kG consecutive elements as 16-byte loads and
// stores where the row allows (phase C layout, d % kG == 0, 16-byte aligned
// row), one element at a time otherwise.
template <class W>
__device__ __forceinline__ void store_row(const float (&v)[W::kN / 256], float* __restrict__ orow,
                                          int d, float sqrtn, float rsq, int dmode,
                                          const float* __restrict__ signs, bool sgn) {
  constexpr int V = W::kN / 256;
  const int t = threadIdx.x;
  if (W::kPhaseC && d % W::kG == 0 && ((uintptr_t)orow & 15) == 0) {
#pragma unroll
    for (int q = 0; q < W::kRuns; ++q) {
      const int i0 = W::idx(t, q * W::kG);
      if (i0 >= d) continue;
#pragma unroll
      for (int c4 = 0; c4 < W::kG / 4; ++c4) {
        const float* vv = v + q * W::kG + 4 * c4;
        float4 o = make_float4(whtr::div_sqrtn(vv[0], sqrtn, rsq, dmode),
                               whtr::div_sqrtn(vv[1], sqrtn, rsq, dmode),
                               whtr::div_sqrtn(vv[2], sqrtn, rsq, dmode),
                               whtr::div_sqrtn(vv[3], sqrtn, rsq, dmode));
        if (sgn) {
          const float4 sg = __ldg(reinterpret_cast<const float4*>(signs + i0) + c4);
          o = make_float4(__fmul_rn(o.x, sg.x), __fmul_rn(o.y, sg.y), __fmul_rn(o.z, sg.z),
                          __fmul_rn(o.w, sg.w));
        }
        reinterpret_cast<float4*>(orow + i0)[c4] = o;
      }
    }
    return;
  }
#pragma unroll
  for (int j = 0; j < V; ++j) {
    const int i = W::idx(t, j);
    if (i < d) {
      float o = whtr::div_sqrtn(v[j], sqrtn, rsq, dmode);
      if (sgn) o = __fmul_rn(o, __ldg(signs + i));
      orow[i] = o;
    }
  }
}

template <int BITS, int KIND, int V>
__global__ void __launch_bounds__(256) hdequant_fast_kernel(
    const uint8_t* __restrict__ packed, const float* __restrict__ scales, int d, float sqrtn,
    float rsq, int dmode, const float* __restrict__ signs, int block, float* __restrict__ out) {
  using W = whtr::Row<V>;
  extern __shared__ __align__(16) float srow[];
  const int64_t r = blockIdx.x;
  const int64_t e0 = r * (int64_t)d;
  const int t = threadIdx.x;
  // scale of element i of the row: scales[(e0 + i) / block]; the row's
  // first block and its offset in it, so the per-element index is 32-bit
  const int64_t b0 = e0 / block;
  const int off = (int)(e0 - b0 * block);
  const float* srow_s = scales + b0;
  const int bshift = (block & (block - 1)) == 0 ? __ffs(block) - 1 : -1;
  float v[V];
  constexpr int RB = W::kG * BITS / 8;  // bytes of one run's codes
  if (W::kPhaseC && BITS <= 8 && d % W::kG == 0 && (e0 * BITS / 8) % RB == 0 &&
      ((uintptr_t)packed % RB) == 0) {
    // each run's codes in one load, decoded in registers, then to the
    // phase-A layout through shared memory
#pragma unroll
    for (int q = 0; q < W::kRuns; ++q) {
      const int i0 = W::idx(t, q * W::kG);
      uint64_t word = 0;
      if (i0 < d) {
        const uint8_t* p = packed + (e0 + i0) * BITS / 8;
        if constexpr (RB == 16) {
          // 16 int8 codes: the low 8 here; the run loop below reads the rest
          word = __ldg(reinterpret_cast<const unsigned long long*>(p));
        } else if constexpr (RB == 8) {
          word = __ldg(reinterpret_cast<const unsigned long long*>(p));
        } else if constexpr (RB == 4) {
          word = __ldg(reinterpret_cast<const uint32_t*>(p));
        } else if constexpr (RB == 2) {
          word = __ldg(reinterpret_cast<const uint16_t*>(p));
        } else {
          word = __ldg(p);
        }
      }
      // a run lies inside one scale block when blocks are whole runs and
      // the row starts on a run boundary of its blocks: one scale load
      const bool run_blk = block % W::kG == 0 && off % W::kG == 0;
      const int k0 = off + i0;
      const float sc0 = (run_blk && i0 < d)
                            ? __ldg(srow_s + (bshift >= 0 ? (k0 >> bshift) : k0 / block))
                            : 0.0f;
#pragma unroll
      for (int c = 0; c < W::kG; ++c) {
        float a = 0.0f;
        if (i0 < d) {
          const int k = off + i0 + c;
          const float sc =
              run_blk ? sc0 : __ldg(srow_s + (bshift >= 0 ? (k >> bshift) : k / block));
          uint32_t raw;
          if constexpr (RB == 16) {
            raw = c < 8 ? (uint32_t)(word >> (8 * c)) & 0xffu
                        : (uint32_t)__ldg(packed + (e0 + i0 + c));
          } else {
            raw = (uint32_t)(word >> (c * BITS)) & ((1u << BITS) - 1u);
          }
          a = dequant_code<BITS, KIND>(raw, sc);
        }
        v[q * W::kG + c] = a;
      }
    }
    if constexpr (W::kPhaseC) W::from_runs(v, srow);
  } else {
#pragma unroll
    for (int j = 0; j < V; ++j) {
      const int i = W::idxA(t, j);
      float a = 0.0f;
      if (i < d) {
        const int k = off + i;
        const float sc = __ldg(srow_s + (bshift >= 0 ? (k >> bshift) : k / block));
        a = dequant_code<BITS, KIND>(raw_code<BITS>(packed, e0 + i), sc);
      }
      v[j] = a;
    }
  }
  W::transform(v, srow);
  store_row<W>(v, out + e0, d, sqrtn, rsq, dmode, signs, true);
}

template <int V>
__global__ void __launch_bounds__(256, V <= 32 ? 4 : 1) hrows_fast_kernel(const float* __restrict__ x, int d,
                                                         float sqrtn, float rsq, int dmode,
                                                         const float* __restrict__ signs,
                                                         bool inverse, float* __restrict__ out) {
  using W = whtr::Row<V>;
  extern __shared__ __align__(16) float srow[];
  const int64_t r = blockIdx.x;
  const float* xr = x + r * d;
  const int t = threadIdx.x;
  float v[V];
  if (W::kPhaseC && d % W::kG == 0 && ((uintptr_t)xr & 15) == 0) {
    // the row in runs of kG consecutive elements (16-byte loads), then to
    // the phase-A layout through shared memory
#pragma unroll
    for (int q = 0; q < W::kRuns; ++q) {
      const int i0 = W::idx(t, q * W::kG);
#pragma unroll
      for (int c4 = 0; c4 < W::kG / 4; ++c4) {
        float4 a = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (i0 < d) {
          a = __ldg(reinterpret_cast<const float4*>(xr + i0) + c4);
          if (!inverse) {
            const float4 sg = __ldg(reinterpret_cast<const float4*>(signs + i0) + c4);
            a = make_float4(__fmul_rn(a.x, sg.x), __fmul_rn(a.y, sg.y), __fmul_rn(a.z, sg.z),
                            __fmul_rn(a.w, sg.w));
          }
        }
        v[q * W::kG + 4 * c4] = a.x;
        v[q * W::kG + 4 * c4 + 1] = a.y;
        v[q * W::kG + 4 * c4 + 2] = a.z;
        v[q * W::kG + 4 * c4 + 3] = a.w;
      }
    }
    if constexpr (W::kPhaseC) W::from_runs(v, srow);
  } else {
#pragma unroll
    for (int j = 0; j < V; ++j) {
      const int i = W::idxA(t, j);
      float a = i < d ? __ldg(xr + i) : 0.0f;
      if (!inverse && i < d) a = __fmul_rn(a, __ldg(signs + i));
      v[j] = a;
    }
  }
  W::transform(v, srow);  // ends with __syncthreads: in-place x == out is safe
  store_row<W>(v, out + r * d, d, sqrtn, rsq, dmode, signs, inverse);
}

// ── pipelined row transform ──────────────────────────────────────────────────
// Persistent CTAs (a few per SM) walk rows r, r + grid, ...; one thread
// requests the next row as a single bulk copy (cp.async.bulk global ->
// shared, completion on an mbarrier, no multicast) while the CTA transforms
// the current one, so each row's DRAM latency is hidden behind the previous
// row's work.  The row buffer doubles as the transform's scratch once its
// values are in registers.  Waits are bounded (2 s of %globaltimer); on
// expiry the kernel records code 7 in the library's error word, waits
// (bounded) for its other copy in flight and returns.
constexpr int kErrRowLoad = 7;  // error-word code of a row copy that never landed

__device__ __forceinline__ uint32_t sm_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void row_bar_init(uint64_t* b) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(sm_addr(b)));
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void row_copy(float* dst, const float* src, uint32_t bytes,
                                         uint64_t* b) {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  asm volatile(
      "{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
          sm_addr(b)),
      "r"(bytes)
      : "memory");
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          sm_addr(dst)),
      "l"(src), "r"(bytes), "r"(sm_addr(b))
      : "memory");
}
__device__ __forceinline__ bool row_wait(uint64_t* b, uint32_t parity) {
  uint64_t t0;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  for (uint32_t i = 0; i < (1u << 24); ++i) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(sm_addr(b)), "r"(parity)
        : "memory");
    if (ok) return true;
    if ((i & 15) == 15) {
      uint64_t t1;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t1));
      if (t1 - t0 > 2000000000ull) break;
    }
  }
  return false;
}

template <int V>
__global__ void __launch_bounds__(256, 3) hrows_pipe_kernel(const float* __restrict__ x,
                                                           int64_t rows, int d, float sqrtn,
                                                           float rsq, int dmode,
                                                           const float* __restrict__ signs,
                                                           bool inverse, float* __restrict__ out,
                                                           int* __restrict__ err) {
  using W = whtr::Row<V>;
  static_assert(W::kPhaseC, "runs layout");
  extern __shared__ __align__(128) float sm[];
  __shared__ __align__(8) uint64_t bar[2];
  const int t = threadIdx.x;
  const uint32_t bytes = (uint32_t)d * 4u;
  if (t == 0) {
    row_bar_init(&bar[0]);
    row_bar_init(&bar[1]);
  }
  __syncthreads();
  int64_t r = blockIdx.x;
  if (t == 0 && r < rows) row_copy(sm, x + r * d, bytes, &bar[0]);
  for (int i = 0; r < rows; ++i, r += gridDim.x) {
    const int cur = i & 1;
    const int64_t rn = r + gridDim.x;
    // `next` was the previous row's scratch, released by the transform's
    // closing barrier
    float* const mine = sm + cur * W::kSmemFloats;
    float* const next = sm + (cur ^ 1) * W::kSmemFloats;
    if (t == 0 && rn < rows) row_copy(next, x + rn * d, bytes, &bar[cur ^ 1]);
    const bool ok = __syncthreads_and(row_wait(&bar[cur], (i >> 1) & 1));
    if (!ok) {
      if (t == 0) {
        if (err) atomicCAS(err, 0, kErrRowLoad);
        if (rn < rows) row_wait(&bar[cur ^ 1], ((i + 1) >> 1) & 1);
      }
      return;
    }
    float v[V];
#pragma unroll
    for (int j = 0; j < V; ++j) {
      const int k = W::idxA(t, j);
      v[j] = inverse ? mine[k] : __fmul_rn(mine[k], __ldg(signs + k));
    }
    W::transform(v, mine);  // opens and closes with __syncthreads
    store_row<W>(v, out + r * d, d, sqrtn, rsq, dmode, signs, inverse);
  }
}

// ── host side ────────────────────────────────────────────────────────────────
constexpr int kMaxHadamardN = 32768;

// How the register transforms divide by fl32(sqrt(hn)) (whtr::div_sqrtn):
// an exact reciprocal product for even powers of two, Markstein's corrected
// product where it was checked equal to the IEEE quotient for every finite
// float, else the IEEE division.
int div_mode(int64_t hn) {
  int l = 0;
  while ((int64_t)1 << l < hn) ++l;
  if (l % 2 == 0) return 1;
  return (l >= 3 && l <= 15) ? 2 : 0;
}

// V of the register-resident transform for row length hn, or 0
int wht_fast_v(int64_t hn) {
  switch (hn) {
    case 2048: return 8;
    case 4096: return 16;
    case 8192: return 32;
    case 16384: return 64;
  }
  return 0;
}

bool pow2(int64_t v) { return v > 0 && (v & (v - 1)) == 0; }
int64_t pow2ceil(int64_t d) {
  int64_t n = 1;
  while (n < d) n <<= 1;
  return n;
}
bool vec_block(int block) { return block >= 8 && block <= 256 && pow2(block); }

int grid_for(int64_t work_threads, int threads = 256) {
  int64_t g = cdiv(work_threads, threads);
  int64_t cap = (int64_t)kSMs * 16;
  if (g > cap) g = cap;
  return (int)(g < 1 ? 1 : g);
}

bool valid_dtype(int bits, int kind) {
  if (kind == MXB_KIND_FLOAT) return bits == 4;
  if (kind == MXB_KIND_INT) return bits == 1 || bits == 2 || bits == 4 || bits == 8;
  return false;
}

bool aligned(const void* p, size_t a) { return ((uintptr_t)p % a) == 0; }

// Launch the base quantizer on a flat input.
template <typename InT, int BITS, int MODE>
int quant_flat(const InT* x, int64_t n, int block, uint8_t* packed, float* scales,
               void* ws, size_t ws_bytes, cudaStream_t st) {
  const int64_t nb = cdiv(n, block);
  const size_t store_align = BITS == 16 ? 16 : (BITS == 8 ? 8 : BITS / 1);
  const bool out_ok = aligned(packed, store_align < 1 ? 1 : store_align);
  if (vec_block(block) && out_ok) {
    const bool vec = aligned(x, 16);
    // 16 elements per lane where the block allows: the per-block shuffles
    // and scale arithmetic are shared by twice the elements (measured at 2^26
    // elements: int4d 0.77 -> 0.85 of HBM from fp32, 0.43 -> 0.56 from bf16)
    if (sizeof(InT) == 2 && block % 32 == 0)
      quant_vec_kernel<InT, BITS, MODE, 32><<<grid_for(nb * (block / 32)), 256, 0, st>>>(
          x, n, block, nb, vec, packed, scales);
    else if (block % 16 == 0)
      quant_vec_kernel<InT, BITS, MODE, 16><<<grid_for(nb * (block / 16)), 256, 0, st>>>(
          x, n, block, nb, vec, packed, scales);
    else
      quant_vec_kernel<InT, BITS, MODE><<<grid_for(nb * (block / 8)), 256, 0, st>>>(
          x, n, block, nb, vec, packed, scales);
    MXB_LAUNCH_CHECK();
    return MXB_OK;
  }
  if (BITS == 16 && !aligned(packed, 4)) return MXB_E_ALIGN;
  if (ws == nullptr || ws_bytes < (size_t)nb * sizeof(float)) return MXB_E_WORKSPACE;
  float* muls = static_cast<float*>(ws);
  quant_scales_kernel<InT, BITS, MODE><<<grid_for(nb * 32), 256, 0, st>>>(x, n, block, nb,
                                                                          scales, muls);
  MXB_LAUNCH_CHECK();
  const int per = BITS == 16 ? 2 : 8 / BITS;
  const int64_t ncodes = nb * block;
  const int64_t nwords = cdiv(ncodes, per);
  quant_pack_kernel<InT, BITS, MODE><<<grid_for(nwords), 256, 0, st>>>(x, n, block, ncodes,
                                                                      nwords, muls, packed);
  MXB_LAUNCH_CHECK();
  return MXB_OK;
}

template <typename InT, int BITS, int MODE>
int quant_dispatch(const InT* x, int64_t n, int64_t row_len, int variant, int block,
                   const float* signs, uint8_t* packed, float* scales, void* ws,
                   size_t ws_bytes, cudaStream_t st) {
  if (variant == MXB_VAR_BASE)
    return quant_flat<InT, BITS, MODE>(x, n, block, packed, scales, ws, ws_bytes, st);
  // Hadamard variant
  const int64_t d = row_len;
  const int64_t hn = pow2ceil(d);
  if (d <= 0 || n % d != 0 || hn > kMaxHadamardN) return MXB_E_SHAPE;
  if (signs == nullptr) return MXB_E_ARG;
  const int64_t rows = n / d;
  const float sqrtn = (float)sqrt((double)hn);
  const size_t smem = (size_t)hn * sizeof(float);
  auto kern = hquant_kernel<InT, BITS, MODE>;
  MXB_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    kMaxHadamardN * (int)sizeof(float)));
  const bool fuse = vec_block(block) && d % block == 0 && aligned(packed, 8);
  const size_t rot_bytes = ((size_t)n * sizeof(float) + 255) & ~(size_t)255;
  if (!fuse && (ws == nullptr || ws_bytes < rot_bytes)) return MXB_E_WORKSPACE;
  float* rot = fuse ? nullptr : static_cast<float*>(ws);
  const int fv = wht_fast_v(hn);
  if (fv) {
    auto launch_fast = [&](auto kf, int V) -> int {
      const size_t fs = ((size_t)hn + (size_t)(hn / 256) * (256 / V)) * sizeof(float);
      MXB_CUDA_TRY(cudaFuncSetAttribute(kf, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)fs));
      MXB_CUDA_TRY(cudaFuncSetAttribute(kf, cudaFuncAttributePreferredSharedMemoryCarveout,
                                        (int)cudaSharedmemCarveoutMaxShared));
      kf<<<(unsigned)rows, 256, fs, st>>>(x, (int)d, sqrtn, 1.0f / sqrtn, div_mode(hn), signs,
                                          block, fuse, packed, scales, rot);
      MXB_LAUNCH_CHECK();
      return MXB_OK;
    };
    int rc;
    switch (fv) {
      case 8: rc = launch_fast(hquant_fast_kernel<InT, BITS, MODE, 8>, 8); break;
      case 16: rc = launch_fast(hquant_fast_kernel<InT, BITS, MODE, 16>, 16); break;
      case 32: rc = launch_fast(hquant_fast_kernel<InT, BITS, MODE, 32>, 32); break;
      default: rc = launch_fast(hquant_fast_kernel<InT, BITS, MODE, 64>, 64); break;
    }
    if (rc != MXB_OK || fuse) return rc;
  } else {
    kern<<<(unsigned)rows, 256, smem, st>>>(x, (int)d, (int)hn, sqrtn, signs, block, fuse,
                                            packed, scales, rot);
    MXB_LAUNCH_CHECK();
    if (fuse) return MXB_OK;
  }
  return quant_flat<float, BITS, MODE>(rot, n, block, packed, scales,
                                       static_cast<char*>(ws) + rot_bytes,
                                       ws_bytes - rot_bytes, st);
}

template <typename InT>
int quant_by_dtype(const InT* x, int64_t n, int64_t row_len, int bits, int kind, int variant,
                   int block, const float* signs, uint8_t* packed, float* scales, void* ws,
                   size_t wsb, cudaStream_t st) {
  if (kind == MXB_KIND_FLOAT)
    return quant_dispatch<InT, 4, Q_FLOAT4>(x, n, row_len, variant, block, signs, packed,
                                            scales, ws, wsb, st);
  switch (bits) {
    case 1: return quant_dispatch<InT, 1, Q_INT_RECIP>(x, n, row_len, variant, block, signs, packed, scales, ws, wsb, st);
    case 2: return quant_dispatch<InT, 2, Q_INT_RECIP>(x, n, row_len, variant, block, signs, packed, scales, ws, wsb, st);
    case 4: return quant_dispatch<InT, 4, Q_INT_RECIP>(x, n, row_len, variant, block, signs, packed, scales, ws, wsb, st);
    case 8: return quant_dispatch<InT, 8, Q_INT_RECIP>(x, n, row_len, variant, block, signs, packed, scales, ws, wsb, st);
  }
  return MXB_E_DTYPE;
}

template <int BITS, int KIND>
int dequant_launch(const uint8_t* packed, const float* scales, int64_t n, int64_t row_len,
                   int variant, int block, const float* signs, float* out, cudaStream_t st) {
  if (variant == MXB_VAR_H) {
    const int64_t d = row_len;
    const int64_t hn = pow2ceil(d);
    if (d <= 0 || n % d != 0 || hn > kMaxHadamardN) return MXB_E_SHAPE;
    if (signs == nullptr) return MXB_E_ARG;
    const float sqrtn = (float)sqrt((double)hn);
    const int fv = wht_fast_v(hn);
    if (fv) {
      auto launch_fast = [&](auto kf, int V) -> int {
        const size_t fs = ((size_t)hn + (size_t)(hn / 256) * (256 / V)) * sizeof(float);
        MXB_CUDA_TRY(cudaFuncSetAttribute(kf, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)fs));
        kf<<<(unsigned)(n / d), 256, fs, st>>>(packed, scales, (int)d, sqrtn, 1.0f / sqrtn,
                                               div_mode(hn), signs, block, out);
        MXB_LAUNCH_CHECK();
        return MXB_OK;
      };
      switch (fv) {
        case 8: return launch_fast(hdequant_fast_kernel<BITS, KIND, 8>, 8);
        case 16: return launch_fast(hdequant_fast_kernel<BITS, KIND, 16>, 16);
        case 32: return launch_fast(hdequant_fast_kernel<BITS, KIND, 32>, 32);
        default: return launch_fast(hdequant_fast_kernel<BITS, KIND, 64>, 64);
      }
    }
    auto kern = hdequant_kernel<BITS, KIND>;
    MXB_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      kMaxHadamardN * (int)sizeof(float)));
    kern<<<(unsigned)(n / d), 256, hn * sizeof(float), st>>>(
        packed, scales, (int)d, (int)hn, sqrtn, signs, block, out);
    MXB_LAUNCH_CHECK();
    return MXB_OK;
  }
  const size_t in_align = BITS == 16 ? 16 : (BITS == 8 ? 8 : (BITS == 4 ? 4 : (BITS == 2 ? 2 : 1)));
  if (block % 8 == 0 && aligned(packed, in_align) && aligned(out, 16)) {
    // Measured at 2^26 elements (fraction of HBM copy bandwidth): the
    // warp-chunk kernel reaches int1/int2/int4/int8/float4 0.84/0.84/0.82/
    // 0.85/0.82, against 0.53 (8 elements per lane) and 0.75-0.79 (4 per
    // lane) for the per-lane kernels, which remain for 16-bit codes and for
    // packed buffers not 4-byte aligned.
#ifndef MXB_DQ8_MASK
#define MXB_DQ8_MASK 0x2  // bit 0: float4, bit 1: int1 take the 8-element kernel
#endif
    constexpr bool v8 = (KIND == MXB_KIND_FLOAT && (MXB_DQ8_MASK & 1)) ||
                        (KIND == MXB_KIND_INT && BITS == 1 && (MXB_DQ8_MASK & 2)) ||
                        (KIND == MXB_KIND_INT && BITS == 2 && (MXB_DQ8_MASK & 4)) ||
                        (KIND == MXB_KIND_INT && BITS == 4 && (MXB_DQ8_MASK & 8)) ||
                        (KIND == MXB_KIND_INT && BITS == 8 && (MXB_DQ8_MASK & 16)) ||
                        (KIND == MXB_KIND_INT && BITS == 16 && (MXB_DQ8_MASK & 32));
#ifndef MXB_DQW_MASK
#define MXB_DQW_MASK 0xf  // bit per width (1, 2, 4, 8 bits) taking the warp-chunk kernel
#endif
    constexpr bool warp = BITS <= 8 && ((MXB_DQW_MASK >> (BITS == 1 ? 0 : BITS == 2 ? 1 :
                                                           BITS == 4 ? 2 : 3)) & 1);
    if (warp && aligned(packed, 4))
      dequant_warp_kernel<(BITS <= 8 ? BITS : 8), KIND><<<grid_for(cdiv(n, 32)), 256, 0, st>>>(
          packed, scales, n, block, out);
    else if (v8)
      dequant_vec8_kernel<BITS, KIND><<<grid_for(cdiv(n, 16)), 256, 0, st>>>(packed, scales, n,
                                                                            block, out);
    else
      dequant_vec_kernel<BITS, KIND><<<grid_for(cdiv(n, 16)), 256, 0, st>>>(packed, scales, n,
                                                                            block, out);
  } else {
    dequant_generic_kernel<BITS, KIND><<<grid_for(n), 256, 0, st>>>(packed, scales, n, block,
                                                                    out);
  }
  MXB_LAUNCH_CHECK();
  return MXB_OK;
}

// dequantize + ReLU, and SiLU(gate) * up: the warp-chunk kernels where the
// block is a multiple of 8 and the pointers are aligned, else per element.
template <int BITS, int KIND>
int dequant_relu_launch(const uint8_t* p, const float* s, int64_t n, int block, float* out,
                        cudaStream_t st) {
  if (BITS <= 8 && block % 8 == 0 && aligned(p, 4) && aligned(out, 16))
    dequant_warp_kernel<(BITS <= 8 ? BITS : 8), KIND, ACT_RELU>
        <<<grid_for(cdiv(n, 32)), 256, 0, st>>>(p, s, n, block, out);
  else
    dequant_generic_kernel<BITS, KIND, ACT_RELU><<<grid_for(n), 256, 0, st>>>(p, s, n, block, out);
  MXB_LAUNCH_CHECK();
  return MXB_OK;
}

template <int BITS, int KIND>
int silu_mul_launch(const uint8_t* gp, const float* gs, const uint8_t* up, const float* us,
                    int64_t n, int block, float* out, cudaStream_t st) {
  if (BITS <= 8 && block % 8 == 0 && aligned(gp, 4) && aligned(up, 4) && aligned(out, 16))
    silu_mul_warp_kernel<(BITS <= 8 ? BITS : 8), KIND>
        <<<grid_for(cdiv(n, 32)), 256, 0, st>>>(gp, gs, up, us, n, block, out);
  else
    silu_mul_generic_kernel<BITS, KIND><<<grid_for(n), 256, 0, st>>>(gp, gs, up, us, n, block, out);
  MXB_LAUNCH_CHECK();
  return MXB_OK;
}

}  // namespace

// Used by the matmul's requantization.
int mxb_requant_f32(const float* c, int64_t n, int block, int out_bits, void* packed,
                    float* scales, void* ws, size_t wsb, cudaStream_t st) {
  uint8_t* p = static_cast<uint8_t*>(packed);
  switch (out_bits) {
    case 2: return quant_flat<float, 2, Q_INT_DIV>(c, n, block, p, scales, ws, wsb, st);
    case 4: return quant_flat<float, 4, Q_INT_DIV>(c, n, block, p, scales, ws, wsb, st);
    case 8: return quant_flat<float, 8, Q_INT_DIV>(c, n, block, p, scales, ws, wsb, st);
    case 16: return quant_flat<float, 16, Q_INT_DIV>(c, n, block, p, scales, ws, wsb, st);
  }
  return MXB_E_DTYPE;
}

size_t mxb_requant_workspace_size(int64_t n, int block) {
  return vec_block(block) ? 0 : (size_t)cdiv(n, block) * sizeof(float);
}

static thread_local char g_last_error[256] = "";
static std::atomic<unsigned long long> g_launches{0};

void mxb_count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

void mxb_set_cuda_error(cudaError_t e) {
  strncpy(g_last_error, cudaGetErrorString(e), sizeof(g_last_error) - 1);
}

extern "C" {

int mxb_version(void) { return 100; }

const char* mxb_last_error(void) { return g_last_error; }

uint64_t mxb_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

size_t mxb_packed_bytes(int64_t n, int bits, int block) {
  if (n < 0 || block <= 0) return 0;
  const int64_t codes = cdiv(n, block) * block;
  if (bits == 16) return (size_t)cdiv(codes, 2) * 4;
  if (bits != 1 && bits != 2 && bits != 4 && bits != 8) return 0;
  return (size_t)cdiv(codes * bits, 8);
}

size_t mxb_quantize_workspace_size(int64_t n, int64_t row_len, int bits, int kind, int variant,
                                   int block) {
  (void)bits; (void)kind;
  if (n <= 0 || block <= 0) return 0;
  size_t flat = vec_block(block) ? 0 : (size_t)cdiv(n, block) * sizeof(float);
  if (variant != MXB_VAR_H) return flat;
  if (vec_block(block) && row_len > 0 && row_len % block == 0) return 0;
  return (((size_t)n * sizeof(float) + 255) & ~(size_t)255) + flat;
}

size_t mxb_dynamic_quantize_workspace_size(int64_t n, int64_t block) {
  if (n <= 0 || block <= 0 || block > INT32_MAX) return 0;
  return vec_block((int)block) ? 0 : (size_t)cdiv(n, block) * sizeof(float);
}

// Per-token / per-tensor quantize: scale = max(amax, 1e-12) / max_int by
// true division, codes = round-half-even(x / scale) (the matmul
// requantization's arithmetic), over flat blocks of any length.
int mxb_dynamic_quantize(const void* x, int x_dtype, int64_t n, int64_t block, int bits,
                         void* packed, float* scales, void* workspace, size_t workspace_bytes,
                         void* stream) {
  if (bits != 2 && bits != 4 && bits != 8 && bits != 16) return MXB_E_DTYPE;
  if (n < 0 || block <= 0 || block > INT32_MAX) return MXB_E_SHAPE;
  if (n == 0) return MXB_OK;
  if (!x || !packed || !scales) return MXB_E_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t* p = static_cast<uint8_t*>(packed);
  const int b = (int)block;
  if (x_dtype == MXB_F32) {
    const float* xf = static_cast<const float*>(x);
    switch (bits) {
      case 2: return quant_flat<float, 2, Q_INT_DIV>(xf, n, b, p, scales, workspace, workspace_bytes, st);
      case 4: return quant_flat<float, 4, Q_INT_DIV>(xf, n, b, p, scales, workspace, workspace_bytes, st);
      case 8: return quant_flat<float, 8, Q_INT_DIV>(xf, n, b, p, scales, workspace, workspace_bytes, st);
      default: return quant_flat<float, 16, Q_INT_DIV>(xf, n, b, p, scales, workspace, workspace_bytes, st);
    }
  }
  if (x_dtype == MXB_BF16) {
    const __nv_bfloat16* xb = static_cast<const __nv_bfloat16*>(x);
    switch (bits) {
      case 2: return quant_flat<__nv_bfloat16, 2, Q_INT_DIV>(xb, n, b, p, scales, workspace, workspace_bytes, st);
      case 4: return quant_flat<__nv_bfloat16, 4, Q_INT_DIV>(xb, n, b, p, scales, workspace, workspace_bytes, st);
      case 8: return quant_flat<__nv_bfloat16, 8, Q_INT_DIV>(xb, n, b, p, scales, workspace, workspace_bytes, st);
      default: return quant_flat<__nv_bfloat16, 16, Q_INT_DIV>(xb, n, b, p, scales, workspace, workspace_bytes, st);
    }
  }
  return MXB_E_DTYPE;
}

int mxb_quantize(const void* x, int x_dtype, int64_t n, int64_t row_len, int bits, int kind,
                 int variant, int block, const float* signs, void* packed, float* scales,
                 void* workspace, size_t workspace_bytes, void* stream) {
  if (!valid_dtype(bits, kind)) return MXB_E_DTYPE;
  if (variant != MXB_VAR_BASE && variant != MXB_VAR_H) return MXB_E_DTYPE;
  if (n < 0 || block <= 0) return MXB_E_SHAPE;
  if (n == 0) return MXB_OK;
  if (!x || !packed || !scales) return MXB_E_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t* p = static_cast<uint8_t*>(packed);
  if (x_dtype == MXB_F32)
    return quant_by_dtype<float>(static_cast<const float*>(x), n, row_len, bits, kind, variant,
                                 block, signs, p, scales, workspace, workspace_bytes, st);
  if (x_dtype == MXB_BF16)
    return quant_by_dtype<__nv_bfloat16>(static_cast<const __nv_bfloat16*>(x), n, row_len,
                                         bits, kind, variant, block, signs, p, scales,
                                         workspace, workspace_bytes, st);
  return MXB_E_DTYPE;
}

int mxb_dequantize(const void* packed, const float* scales, int64_t n, int64_t row_len,
                   int bits, int kind, int variant, int block, const float* signs, float* out,
                   void* stream) {
  if (!(valid_dtype(bits, kind) || (bits == 16 && kind == MXB_KIND_INT))) return MXB_E_DTYPE;
  if (variant != MXB_VAR_BASE && variant != MXB_VAR_H) return MXB_E_DTYPE;
  if (n < 0 || block <= 0) return MXB_E_SHAPE;
  if (n == 0) return MXB_OK;
  if (!packed || !scales || !out) return MXB_E_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const uint8_t* p = static_cast<const uint8_t*>(packed);
  if (kind == MXB_KIND_FLOAT)
    return dequant_launch<4, MXB_KIND_FLOAT>(p, scales, n, row_len, variant, block, signs, out, st);
  switch (bits) {
    case 1: return dequant_launch<1, MXB_KIND_INT>(p, scales, n, row_len, variant, block, signs, out, st);
    case 2: return dequant_launch<2, MXB_KIND_INT>(p, scales, n, row_len, variant, block, signs, out, st);
    case 4: return dequant_launch<4, MXB_KIND_INT>(p, scales, n, row_len, variant, block, signs, out, st);
    case 8: return dequant_launch<8, MXB_KIND_INT>(p, scales, n, row_len, variant, block, signs, out, st);
    case 16: return dequant_launch<16, MXB_KIND_INT>(p, scales, n, row_len, variant, block, signs, out, st);
  }
  return MXB_E_DTYPE;
}

int mxb_dequantize_relu(const void* packed, const float* scales, int64_t n, int bits, int kind,
                        int block, float* out, void* stream) {
  if (!(valid_dtype(bits, kind) || (bits == 16 && kind == MXB_KIND_INT))) return MXB_E_DTYPE;
  if (n < 0 || block <= 0) return MXB_E_SHAPE;
  if (n == 0) return MXB_OK;
  if (!packed || !scales || !out) return MXB_E_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const uint8_t* p = static_cast<const uint8_t*>(packed);
  if (kind == MXB_KIND_FLOAT) return dequant_relu_launch<4, MXB_KIND_FLOAT>(p, scales, n, block, out, st);
  switch (bits) {
    case 1: return dequant_relu_launch<1, MXB_KIND_INT>(p, scales, n, block, out, st);
    case 2: return dequant_relu_launch<2, MXB_KIND_INT>(p, scales, n, block, out, st);
    case 4: return dequant_relu_launch<4, MXB_KIND_INT>(p, scales, n, block, out, st);
    case 8: return dequant_relu_launch<8, MXB_KIND_INT>(p, scales, n, block, out, st);
    case 16: return dequant_relu_launch<16, MXB_KIND_INT>(p, scales, n, block, out, st);
  }
  return MXB_E_DTYPE;
}

int mxb_dequantize_silu_mul(const void* gate_packed, const float* gate_scales,
                            const void* up_packed, const float* up_scales, int64_t n, int bits,
                            int kind, int block, float* out, void* stream) {
  if (!(valid_dtype(bits, kind) || (bits == 16 && kind == MXB_KIND_INT))) return MXB_E_DTYPE;
  if (n < 0 || block <= 0) return MXB_E_SHAPE;
  if (n == 0) return MXB_OK;
  if (!gate_packed || !gate_scales || !up_packed || !up_scales || !out) return MXB_E_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const uint8_t* g = static_cast<const uint8_t*>(gate_packed);
  const uint8_t* u = static_cast<const uint8_t*>(up_packed);
  if (kind == MXB_KIND_FLOAT)
    return silu_mul_launch<4, MXB_KIND_FLOAT>(g, gate_scales, u, up_scales, n, block, out, st);
  switch (bits) {
    case 1: return silu_mul_launch<1, MXB_KIND_INT>(g, gate_scales, u, up_scales, n, block, out, st);
    case 2: return silu_mul_launch<2, MXB_KIND_INT>(g, gate_scales, u, up_scales, n, block, out, st);
    case 4: return silu_mul_launch<4, MXB_KIND_INT>(g, gate_scales, u, up_scales, n, block, out, st);
    case 8: return silu_mul_launch<8, MXB_KIND_INT>(g, gate_scales, u, up_scales, n, block, out, st);
    case 16: return silu_mul_launch<16, MXB_KIND_INT>(g, gate_scales, u, up_scales, n, block, out, st);
  }
  return MXB_E_DTYPE;
}

int mxb_hadamard_rows(const float* x, int64_t rows, int64_t d, const float* signs, int inverse,
                      float* out, void* stream) {
  if (rows < 0 || d <= 0) return MXB_E_SHAPE;
  if (rows == 0) return MXB_OK;
  if (!x || !signs || !out) return MXB_E_ARG;
  const int64_t hn = pow2ceil(d);
  if (hn > kMaxHadamardN) return MXB_E_SHAPE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const float sqrtn = (float)sqrt((double)hn);
  const int fv = wht_fast_v(hn);
  // pipelined kernel: whole power-of-two rows, 16-byte aligned, enough rows
  // to keep every CTA busy for a few rows
  if ((fv == 16 || fv == 32) && d == hn && ((uintptr_t)x & 15) == 0 &&
      ((uintptr_t)out & 15) == 0 && rows >= 4 * kSMs) {
    auto kp = fv == 16 ? hrows_pipe_kernel<16> : hrows_pipe_kernel<32>;
    const size_t fs = 2 * ((size_t)hn + (size_t)(hn / 256) * (256 / fv)) * sizeof(float);
    MXB_CUDA_TRY(cudaFuncSetAttribute(kp, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)fs));
    MXB_CUDA_TRY(cudaFuncSetAttribute(kp, cudaFuncAttributePreferredSharedMemoryCarveout,
                                      (int)cudaSharedmemCarveoutMaxShared));
    int per_sm = 0;
    MXB_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kp, 256, fs));
    if (per_sm < 1) per_sm = 1;
    const int64_t grid = rows < (int64_t)per_sm * kSMs ? rows : (int64_t)per_sm * kSMs;
    kp<<<(unsigned)grid, 256, fs, st>>>(x, rows, (int)d, sqrtn, 1.0f / sqrtn, div_mode(hn), signs,
                                        inverse != 0, out, device_error_ptr());
    MXB_LAUNCH_CHECK();
    return MXB_OK;
  }
  if (fv) {
    auto launch_fast = [&](auto kf, int V) -> int {
      const size_t fs = ((size_t)hn + (size_t)(hn / 256) * (256 / V)) * sizeof(float);
      MXB_CUDA_TRY(cudaFuncSetAttribute(kf, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)fs));
      MXB_CUDA_TRY(cudaFuncSetAttribute(kf, cudaFuncAttributePreferredSharedMemoryCarveout,
                                        (int)cudaSharedmemCarveoutMaxShared));
      kf<<<(unsigned)rows, 256, fs, st>>>(x, (int)d, sqrtn, 1.0f / sqrtn, div_mode(hn), signs,
                                          inverse != 0, out);
      MXB_LAUNCH_CHECK();
      return MXB_OK;
    };
    switch (fv) {
      case 8: return launch_fast(hrows_fast_kernel<8>, 8);
      case 16: return launch_fast(hrows_fast_kernel<16>, 16);
      case 32: return launch_fast(hrows_fast_kernel<32>, 32);
      default: return launch_fast(hrows_fast_kernel<64>, 64);
    }
  }
  MXB_CUDA_TRY(cudaFuncSetAttribute(hrows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    kMaxHadamardN * (int)sizeof(float)));
  hrows_kernel<<<(unsigned)rows, 256, hn * sizeof(float), st>>>(x, (int)d, (int)hn, sqrtn, signs,
                                                              inverse != 0, out);
  MXB_LAUNCH_CHECK();
  return MXB_OK;
}

}  // extern "C"
