// tcgen05 weight-only GEMM for the prefill regime of mx_linear (M > 16):
//
//   y[m, n] = sum_k x[m, k] * w[k, n],  w = fl(code[k, n] * s[k, n / block])
//   (mxtorch.py:7454-7473; x bf16, W^T [K, N] packed codes + block scales)
//
// The scale varies along K, so it cannot move to the epilogue.  Instead the
// dequantized weight w (exact fp32, the reference's value) is split into
// bf16 planes: hi = bf16(w), mid = bf16(w - hi), |w - hi - mid| <= 2^-18 |w|.
// Parity mode multiplies x (exact in bf16) by both planes with one
// kind::f16 MMA of N = 256 per K slice (the planes are stored back to back
// as one 256-row operand) into hi and mid partial sums that the epilogue
// adds; fast mode uses hi only (N = 128).
//
// One CTA owns a 256 x 128 tile of y (two M=128 accumulators in TMEM that
// share the weight planes):
//   warp 0     TMA producer: x [256 x 64] bf16 (128-byte swizzle) and the
//              packed codes [64 K rows x 128 N] per K step, 3-stage ring;
//   warp 1     TMEM allocation and MMA issue (4 K=16 steps x 2 halves);
//   warps 2-9  transform, two groups of 4 taking alternate K steps (group j
//              fills plane buffer j): each thread dequantizes an 8 (N) x 8 (K)
//              unit of codes and writes the bf16 planes straight into the
//              128-byte swizzled K-major layout; scales are fetched one step
//              ahead.  Then the epilogue (tcgen05.ld -> fp32 y), group j
//              draining accumulator j.
// Included by gemm_tc.cu (shares its device error word).
#pragma once

namespace mxb {
namespace wo {

constexpr int BM = 256, BN = 128, BK = 64;  // BK in bf16 elements (128 bytes)
constexpr int STAGES = 3;
constexpr int kTransWarps = 8;               // two groups of 4
constexpr int kGroupWarps = kTransWarps / 2;
constexpr int kThreads = 64 + 32 * kTransWarps;
constexpr int kAHalf = 128 * BK * 2;      // 16 KB
constexpr int kAStage = 2 * kAHalf;       // 32 KB
constexpr int kPlane = BN * BK * 2;       // 16 KB
constexpr int kCodeStageMax = BK * BN;    // int8: 8 KB
constexpr size_t kBarsBytes = 256;
constexpr size_t kSmemBytes =
    1024 + (size_t)STAGES * kAStage + 2 * 2 * kPlane + (size_t)STAGES * kCodeStageMax + kBarsBytes;

struct Bars {
  uint64_t full[STAGES];   // x + codes of a stage landed
  uint64_t empty[STAGES];  // MMA done with x, transform done with codes
  uint64_t bready[2];      // weight planes j written
  uint64_t bfree[2];       // MMAs reading planes j done
  uint64_t accfull;        // all MMAs done
  uint32_t tmem_base;
};
static_assert(sizeof(Bars) <= kBarsBytes, "barrier block overflows its slot");

__device__ __forceinline__ float small_int_to_float(int c) {
  // exact for |c| < 2^22 (c is a 1..8-bit code here)
  return __fsub_rn(__int_as_float(0x4B400000 + c), 12582912.0f);
}

template <int BITS, int KIND>
__device__ __forceinline__ float wdeq(uint32_t raw, float s) {
  if (KIND == MXB_KIND_FLOAT) return __fmul_rn(f4_grid((int)raw), s);
  if (BITS == 1) return (raw & 1u) ? -s : s;
  return __fmul_rn(small_int_to_float(sext(raw, BITS)), s);
}

template <int BITS>
__device__ __forceinline__ uint64_t lds_codes(const uint8_t* p) {
  if constexpr (BITS == 8) {
    uint2 v = *reinterpret_cast<const uint2*>(p);
    return (uint64_t)v.x | ((uint64_t)v.y << 32);
  } else if constexpr (BITS == 4) {
    return *reinterpret_cast<const uint32_t*>(p);
  } else if constexpr (BITS == 2) {
    return *reinterpret_cast<const uint16_t*>(p);
  } else {
    return *p;
  }
}

__device__ __forceinline__ uint32_t bf16x2_rn(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ float bf16lo_f(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf16hi_f(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// KMAJ: the weight is W [N, K] quantized flat (mx_dynamic_linear's layout,
// scale s[n, k / block]); its code tile arrives K-major, [128 N rows][BK
// codes], which is already the plane's orientation, so the transform reads
// 8 consecutive K codes of one N row instead of transposing.
template <int BITS, int KIND, bool FAST, bool KMAJ>
__global__ void __launch_bounds__(kThreads, 1)
    wonly_tc_kernel(const __grid_constant__ CUtensorMap tmap_x,
                    const __grid_constant__ CUtensorMap tmap_w, const float* __restrict__ ws,
                    int M, int N, int K, int block, float* __restrict__ y) {
  constexpr int kCodeRow = BN * BITS / 8;     // bytes of one K row of the code tile
  constexpr int kCodeRowK = BK * BITS / 8;    // KMAJ: bytes of one N row of the code tile
  constexpr int kCodeStage = BK * kCodeRow;
  // parity: per M half one N = 256 accumulator, columns [0, 128) the hi
  // plane's products and [128, 256) the mid plane's (the planes are stored
  // back to back, so they form one 256-row B operand: each x tile is read
  // once per K slice instead of once per plane); fast: hi only
  constexpr int kAcc = FAST ? BN : 2 * BN;
  constexpr uint32_t kCols = 2 * kAcc;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;                                  // STAGES x [2 halves x 16 KB]
  uint8_t* sP = sA + STAGES * kAStage;                 // 2 buffers x [hi, mid] planes
  uint8_t* sC = sP + 2 * 2 * kPlane;                   // STAGES x code tiles
  Bars* bars = reinterpret_cast<Bars*>(sC + STAGES * kCodeStageMax);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  const int ksteps = K / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1 + kGroupWarps);
    }
    for (int j = 0; j < 2; ++j) {
      mbar_init(&bars->bready[j], kGroupWarps);
      mbar_init(&bars->bfree[j], 1);
    }
    mbar_init(&bars->accfull, 1);
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmap_x);
    prefetch_tmap(&tmap_w);
  }
  if (warp == 1) {
    tmem_alloc(&bars->tmem_base, kCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = bars->tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      for (int ks = 0; ks < ksteps; ++ks) {
        const int s = ks % STAGES, round = ks / STAGES;
        if (round > 0 && !mbar_wait(&bars->empty[s], (round - 1) & 1, kErrTimeoutEmpty)) break;
        mbar_expect_tx(&bars->full[s], kAStage + kCodeStage);
        tma_load_2d(sA + s * kAStage, &tmap_x, &bars->full[s], ks * BK, m0);
        tma_load_2d(sA + s * kAStage + kAHalf, &tmap_x, &bars->full[s], ks * BK, m0 + 128);
        if constexpr (KMAJ)
          tma_load_2d(sC + s * kCodeStageMax, &tmap_w, &bars->full[s], ks * kCodeRowK, n0);
        else
          tma_load_2d(sC + s * kCodeStageMax, &tmap_w, &bars->full[s], n0 * BITS / 8, ks * BK);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc(/*F32*/ 1, /*BF16*/ 1, 0, 0, 128, kAcc);
      for (int ks = 0; ks < ksteps; ++ks) {
        const int s = ks % STAGES, round = ks / STAGES;
        const int j = ks & 1, usej = ks >> 1;
        if (!mbar_wait(&bars->full[s], round & 1, kErrTimeoutFull)) break;
        if (!mbar_wait(&bars->bready[j], usej & 1, kErrTimeoutTmemFull)) break;
        tc_fence_after();
        const uint32_t a0 = smem_u32(sA + s * kAStage);
        const uint32_t phi = smem_u32(sP + (2 * j) * kPlane);
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const uint64_t ad = desc_kmajor_sw128(a0 + h * kAHalf + kk * 32);
            mma_f16(tbase + h * kAcc, ad, desc_kmajor_sw128(phi + kk * 32), idesc,
                    (ks > 0 || kk > 0) ? 1u : 0u);
          }
        }
        mma_commit(&bars->empty[s]);
        mma_commit(&bars->bfree[j]);
      }
      mma_commit(&bars->accfull);
    }
  } else if (KMAJ) {
    // ── transform, K-major codes: thread (n8 = t / 8, k8 = t % 8) takes the
    // 8 K codes k8*8.. of N rows n8*8 + c, c = 0..7 (row order rotated by
    // n8 so the warp's four rows sit in different banks) ──
    const int grp = (warp - 2) >> 2;
    const int t = (threadIdx.x - 64) & 127;
    const int n8 = t >> 3, k8 = t & 7;
    const int nkb = K / block;  // scales per N row (K % block == 0)
    const float* sp = ws + (size_t)(n0 + n8 * 8) * nkb;
    float sc_next[8];
    if (grp < ksteps) {
#pragma unroll
      for (int c = 0; c < 8; ++c)
        sc_next[c] = __ldg(sp + (size_t)c * nkb + (grp * BK + k8 * 8) / block);
    }
    for (int ks = grp; ks < ksteps; ks += 2) {
      const int s = ks % STAGES, round = ks / STAGES;
      const int j = grp, usej = ks >> 1;
      float sc[8];
#pragma unroll
      for (int c = 0; c < 8; ++c) sc[c] = sc_next[c];
      if (ks + 2 < ksteps) {
#pragma unroll
        for (int c = 0; c < 8; ++c)
          sc_next[c] = __ldg(sp + (size_t)c * nkb + ((ks + 2) * BK + k8 * 8) / block);
      }
      if (!mbar_wait_warp(&bars->full[s], round & 1, kErrTimeoutFull)) break;
      uint64_t word[8];
      const uint8_t* cp = sC + s * kCodeStageMax + k8 * BITS;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const int r = n8 * 8 + ((c + n8) & 7);
        word[c] = lds_codes<BITS>(cp + r * kCodeRowK);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->empty[s]);
      if (usej > 0 && !mbar_wait_warp(&bars->bfree[j], (usej - 1) & 1, kErrTimeoutTmemEmpty))
        break;
      uint8_t* phi = sP + (2 * j) * kPlane;
      uint8_t* pmid = sP + (2 * j + 1) * kPlane;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const int cc = (c + n8) & 7;
        const int r = n8 * 8 + cc;  // N row of the plane
        float w[8];
#pragma unroll
        for (int i = 0; i < 8; ++i)
          w[i] = wdeq<BITS, KIND>((uint32_t)(word[c] >> (i * BITS)) & ((1u << BITS) - 1u), sc[cc]);
        uint4 hv, mv;
        uint32_t* h4 = reinterpret_cast<uint32_t*>(&hv);
        uint32_t* m4 = reinterpret_cast<uint32_t*>(&mv);
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          h4[p] = bf16x2_rn(w[2 * p], w[2 * p + 1]);
          if (!FAST)
            m4[p] = bf16x2_rn(__fsub_rn(w[2 * p], bf16lo_f(h4[p])),
                              __fsub_rn(w[2 * p + 1], bf16hi_f(h4[p])));
        }
        const int off = r * 128 + ((k8 ^ (r & 7)) << 4);  // 128-byte swizzle, K-major
        *reinterpret_cast<uint4*>(phi + off) = hv;
        if (!FAST) *reinterpret_cast<uint4*>(pmid + off) = mv;
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->bready[j]);
    }
    // ── epilogue: TMEM -> y ──
    if (mbar_wait_warp(&bars->accfull, 0, kErrTimeoutDone)) {
      tc_fence_after();
      const int q = warp & 3;
      const int h = grp;
      const int m = m0 + h * 128 + q * 32 + lane;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32], rm[32];
        const uint32_t ta = tbase + ((uint32_t)(q * 32) << 16) + h * kAcc + c * 32;
        tmem_ld32(ta, r);
        if (!FAST) tmem_ld32(ta + BN, rm);
        tmem_wait_ld();
        if (!FAST) {
#pragma unroll
          for (int v = 0; v < 32; ++v)
            r[v] = __float_as_uint(__fadd_rn(__uint_as_float(r[v]), __uint_as_float(rm[v])));
        }
        if (m < M) {
          float4* o = reinterpret_cast<float4*>(y + (size_t)m * N + n0 + c * 32);
#pragma unroll
          for (int v = 0; v < 8; ++v)
            o[v] = make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]),
                               __uint_as_float(r[4 * v + 2]), __uint_as_float(r[4 * v + 3]));
        }
      }
    }
  } else {
    // ── transform: two groups of 4 warps take alternate K steps, group j
    // filling plane buffer j; one 8 (N) x 8 (K) unit per thread per step ──
    const int grp = (warp - 2) >> 2;
    const int t = (threadIdx.x - 64) & 127;
    const int n8 = t & 15, k8 = t >> 4;  // n-group (16 of 8 columns), k-group (8 of 8 rows)
    const int nsb = N / block;
    const float* sp = ws + (size_t)(n0 + n8 * 8) / block + (size_t)(k8 * 8) * nsb;
    // When the tile's 128 columns share one scale block (block % 128 == 0)
    // the warp needs only 16 scales per step (its two 8-row K groups): lane
    // l loads row l % 16 and the others read it by shuffle.  Otherwise each
    // thread loads its own 8.  Either way one step ahead.
    const bool one_block = block % BN == 0;
    const int wrow0 = ((t >> 5) << 4);  // first K row of this warp within a step
    const float* sp1 = ws + (size_t)n0 / block + (size_t)(wrow0 + (lane & 15)) * nsb;
    float sc_next[8], s1_next = 0.0f;
    if (grp < ksteps) {
      if (one_block) {
        s1_next = __ldg(sp1 + (size_t)(grp * BK) * nsb);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) sc_next[i] = __ldg(sp + (size_t)(grp * BK + i) * nsb);
      }
    }
    for (int ks = grp; ks < ksteps; ks += 2) {
      const int s = ks % STAGES, round = ks / STAGES;
      const int j = grp, usej = ks >> 1;
      float sc[8];
      if (one_block) {
        const float s1 = s1_next;
        if (ks + 2 < ksteps) s1_next = __ldg(sp1 + (size_t)((ks + 2) * BK) * nsb);
#pragma unroll
        for (int i = 0; i < 8; ++i) sc[i] = __shfl_sync(0xffffffffu, s1, ((lane >> 4) << 3) + i);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) sc[i] = sc_next[i];
        if (ks + 2 < ksteps) {
#pragma unroll
          for (int i = 0; i < 8; ++i) sc_next[i] = __ldg(sp + (size_t)((ks + 2) * BK + i) * nsb);
        }
      }
      if (!mbar_wait_warp(&bars->full[s], round & 1, kErrTimeoutFull)) break;
      uint64_t word[8];
      const uint8_t* cp = sC + s * kCodeStageMax + (k8 * 8) * kCodeRow + n8 * BITS;
#pragma unroll
      for (int i = 0; i < 8; ++i) word[i] = lds_codes<BITS>(cp + i * kCodeRow);
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->empty[s]);
      if (usej > 0 && !mbar_wait_warp(&bars->bfree[j], (usej - 1) & 1, kErrTimeoutTmemEmpty))
        break;
      uint8_t* phi = sP + (2 * j) * kPlane;
      uint8_t* pmid = sP + (2 * j + 1) * kPlane;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        // rotate the column order by n8 so the lanes of a warp store to 8
        // different 16-byte bank groups (r & 7 varies across lanes)
        const int cc = (c + n8) & 7;
        const int r = n8 * 8 + cc;  // N row of the plane
        float w[8];
#pragma unroll
        for (int i = 0; i < 8; ++i)
          w[i] = wdeq<BITS, KIND>((uint32_t)(word[i] >> (cc * BITS)) & ((1u << BITS) - 1u), sc[i]);
        uint4 hv, mv;
        uint32_t* h4 = reinterpret_cast<uint32_t*>(&hv);
        uint32_t* m4 = reinterpret_cast<uint32_t*>(&mv);
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          h4[p] = bf16x2_rn(w[2 * p], w[2 * p + 1]);
          if (!FAST)
            m4[p] = bf16x2_rn(__fsub_rn(w[2 * p], bf16lo_f(h4[p])),
                              __fsub_rn(w[2 * p + 1], bf16hi_f(h4[p])));
        }
        const int off = r * 128 + ((k8 ^ (r & 7)) << 4);  // 128-byte swizzle, K-major
        *reinterpret_cast<uint4*>(phi + off) = hv;
        if (!FAST) *reinterpret_cast<uint4*>(pmid + off) = mv;
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->bready[j]);
    }
    // ── epilogue: TMEM -> y ──
    if (mbar_wait_warp(&bars->accfull, 0, kErrTimeoutDone)) {
      tc_fence_after();
      const int q = warp & 3;
      {
        const int h = grp;  // accumulator (M half) of this warp's group
        const int m = m0 + h * 128 + q * 32 + lane;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t r[32], rm[32];
          const uint32_t ta = tbase + ((uint32_t)(q * 32) << 16) + h * kAcc + c * 32;
          tmem_ld32(ta, r);
          if (!FAST) tmem_ld32(ta + BN, rm);
          tmem_wait_ld();
          if (!FAST) {
#pragma unroll
            for (int v = 0; v < 32; ++v)
              r[v] = __float_as_uint(__fadd_rn(__uint_as_float(r[v]), __uint_as_float(rm[v])));
          }
          if (m < M) {
            float4* o = reinterpret_cast<float4*>(y + (size_t)m * N + n0 + c * 32);
#pragma unroll
            for (int v = 0; v < 8; ++v)
              o[v] = make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]),
                                 __uint_as_float(r[4 * v + 2]), __uint_as_float(r[4 * v + 3]));
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    mbar_wait(&bars->accfull, 0, kErrTimeoutDone);
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tbase, kCols);
  }
}

}  // namespace wo
}  // namespace mxb
