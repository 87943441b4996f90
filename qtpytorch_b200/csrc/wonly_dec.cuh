// tcgen05 weight-only linear for the decode regime of mx_linear (3 <= M <= 32,
// bf16 x, integer codes, scale blocks spanning whole 128-column tiles):
//
//   y[m, n] = sum_k x[m, k] * fl(code[k, n] * s[k, n / block])   (mxtorch.py:7454-7473)
//           ~ sum_k fl(x[m, k] * s[k, nb]) * code[k, n]
//
// With block % 128 == 0 all 128 columns of a tile share one scale per K row,
// so the scale moves onto the (tiny) activation instead of the weight: the
// weight tile only needs its integer codes converted to bf16 (exact for
// 1..8-bit codes), and x' = fl(x * s) is split into two bf16 planes
// hi + mid (|x' - hi - mid| <= 2^-18 |x'|).  Roles are swapped against the
// prefill kernel: the 128 weight columns are the MMA's M (an MN-major
// operand, the codes' own [K][N] order); the two x' planes, each padded to
// MP in {16, 32} token rows, are stacked into one N = 2 * MP operand, so one
// MMA per K slice reads the weight plane once and yields both partial
// products (added in the epilogue).  A tcgen05 MMA with M = 128 costs about
// the same for N = 16..64, so M up to 32 runs at one price.
//
// One CTA owns 128 columns and a K chunk (split-K across blockIdx.y; partial
// sums go to a workspace and are added in split order by a second kernel):
//   warp 0     TMA producer: packed codes [64 K rows x 128 N] per step, ring
//              of STAGES stages;
//   warp 1     TMEM allocation and MMA issue: per step 4 K=16 slices into
//              D[128 x 2 MP] fp32 in TMEM (hi products | mid products);
//   warps 2-9  transform, two groups of 4 taking alternate steps (step ks
//              fills plane buffer ks % kBufs): codes -> bf16 A plane (8 contiguous
//              codes -> one 16-byte chunk of the 128-byte swizzled MN-major
//              layout), x' -> two bf16 B planes with x loaded one step
//              ahead; then group 0 runs the epilogue (tcgen05.ld, one column
//              of y per thread, hi + mid halves added).
// Included by gemm_tc.cu (shares its device error word and helpers).
#pragma once

namespace mxb {
namespace dec {

constexpr int BN = 128, BK = 64;
constexpr int STAGES = 6;
// plane buffers (step ks uses ks % kBufs): 2 measured as fast as 4 for
// M <= 16 and faster at M = 32 (less shared memory: 43 -> 35 us at 4096 x 11008)
constexpr int kBufs = 2;
constexpr int kGroupWarps = 4;
constexpr int kTransWarps = 2 * kGroupWarps;
constexpr int kThreads = 64 + 32 * kTransWarps;
constexpr int kPlaneA = BN * BK * 2;        // 16 KB: two 64-column atoms of 8 KB
constexpr int kAtomA = kPlaneA / 2;
constexpr int kXPlanes = 2;                 // x' = hi + mid
constexpr int kMaxKc = kDecMaxKc;           // K rows per CTA (scales staged in smem)
constexpr int kTmemCols = 64;
constexpr size_t kBarsBytes = 256;

template <int MP>
constexpr int plane_b() { return MP * BK * 2; }  // one x' plane: MP rows x 128 B
template <int BITS>
constexpr int code_stage() { return BK * BN * BITS / 8; }

// dynamic shared memory of a launch with K chunk kc (the scales come last)
template <int BITS, int MP>
constexpr size_t smem_bytes(int kc) {
  return 1024 + kBufs * (kPlaneA + kXPlanes * plane_b<MP>()) +
         (size_t)STAGES * code_stage<BITS>() + kBarsBytes + (size_t)kc * 4;
}

struct Bars {
  uint64_t full[STAGES];   // codes of a stage landed
  uint64_t empty[STAGES];  // transform done reading a stage
  uint64_t bready[kBufs];  // planes b written
  uint64_t bfree[kBufs];   // MMAs reading planes b done
  uint64_t accfull;        // all MMAs done
  uint32_t tmem_base;
};
static_assert(sizeof(Bars) <= kBarsBytes, "barrier block overflows its slot");

// high halves of two floats -> bf16x2 (exact for the small integers here)
__device__ __forceinline__ uint32_t hi_halves(float lo, float hi) {
  return __byte_perm(__float_as_uint(lo), __float_as_uint(hi), 0x7632);
}

// 8 consecutive codes (one row, 8 columns) -> 8 exact bf16 values as uint4.
template <int BITS>
__device__ __forceinline__ uint4 codes8_bf16(const uint8_t* p) {
  uint32_t o[4];
  if constexpr (BITS == 4) {
    // offset binary u = code + 8 placed in the mantissa of bf16 128 (0x4300)
    // reads as 128 + u; one packed bf16 subtraction of 136 leaves the code
    // (exact: small integers).  Byte k of t holds codes 2k (low nibble) and,
    // shifted down in s, 2k + 1.
    const uint32_t t = *reinterpret_cast<const uint32_t*>(p) ^ 0x88888888u;
    const uint32_t s = t >> 4;
    const __nv_bfloat162 bias = __floats2bfloat162_rn(136.0f, 136.0f);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      // result byte 0 = byte k of t, byte 2 = byte k of s (bytes 1, 3 masked)
      const uint32_t sel = (uint32_t)(k | (k << 4) | ((4 + k) << 8) | ((4 + k) << 12));
      const uint32_t x = (__byte_perm(t, s, sel) & 0x000F000Fu) | 0x43004300u;
      __nv_bfloat162 c = __hsub2(*reinterpret_cast<const __nv_bfloat162*>(&x), bias);
      o[k] = *reinterpret_cast<uint32_t*>(&c);
    }
  } else if constexpr (BITS == 8) {
    const uint2 w = *reinterpret_cast<const uint2*>(p);
    const uint32_t ws[2] = {w.x ^ 0x80808080u, w.y ^ 0x80808080u};  // code + 128
    const uint64_t bias = pack2(8388736.0f, 8388736.0f);              // 2^23 + 128
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const float2 c = unpack2(
            fsub2(pack2(__int_as_float(__byte_perm(ws[h], 0x4B000000u, 0x7440 + 2 * k)),
                        __int_as_float(__byte_perm(ws[h], 0x4B000000u, 0x7441 + 2 * k))),
                  bias));
        o[2 * h + k] = hi_halves(c.x, c.y);
      }
  } else {
    const uint32_t w = BITS == 2 ? *reinterpret_cast<const uint16_t*>(p) : *p;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      uint32_t b[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const uint32_t raw = (w >> ((2 * k + e) * BITS)) & ((1u << BITS) - 1u);
        b[e] = BITS == 1 ? ((raw & 1u) ? 0xBF80u : 0x3F80u)  // raw 1 -> -1, raw 0 -> +1
                         : __float_as_uint(wo::small_int_to_float(sext(raw, BITS))) >> 16;
      }
      o[k] = b[0] | (b[1] << 16);
    }
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

template <int BITS, int MP>
__global__ void __launch_bounds__(kThreads)
    wonly_dec_kernel(const __grid_constant__ CUtensorMap tmap_w,
                     const __nv_bfloat16* __restrict__ x, const float* __restrict__ ws, int M,
                     int N, int K, int block, int kc, float* __restrict__ out) {
  constexpr int kCodeRow = BN * BITS / 8;  // bytes of one K row of the code tile
  constexpr int kCodeStage = code_stage<BITS>();
  constexpr int kPlaneB = plane_b<MP>();
  constexpr int kChunks = MP * BK / 8 / 128;  // 8-value x chunks per thread and step (1 or 2)
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;                                  // kBufs x codes plane
  uint8_t* sB = sA + kBufs * kPlaneA;                  // kBufs x 2 x' planes
  uint8_t* sC = sB + kBufs * kXPlanes * kPlaneB;       // STAGES x code tiles
  Bars* bars = reinterpret_cast<Bars*>(sC + STAGES * kCodeStage);
  float* sS = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(bars) + kBarsBytes);  // kc scales

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * BN;
  const int k0 = blockIdx.y * kc;
  const int kn = min(kc, K - k0);
  const int ksteps = kn / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], kGroupWarps);
    }
    for (int j = 0; j < kBufs; ++j) {
      mbar_init(&bars->bready[j], kGroupWarps);
      mbar_init(&bars->bfree[j], 1);
    }
    mbar_init(&bars->accfull, 1);
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) prefetch_tmap(&tmap_w);
  if (warp == 1) {
    tmem_alloc(&bars->tmem_base, kTmemCols);
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
        mbar_expect_tx(&bars->full[s], kCodeStage);
        tma_load_2d(sC + s * kCodeStage, &tmap_w, &bars->full[s], n0 * BITS / 8, k0 + ks * BK);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc =
          make_idesc(/*F32*/ 1, /*BF16*/ 1, /*A MN-major*/ 1, 0, BN, kXPlanes * MP);
      for (int ks = 0; ks < ksteps; ++ks) {
        const int j = ks % kBufs, usej = ks / kBufs;
        if (!mbar_wait(&bars->bready[j], usej & 1, kErrTimeoutTmemFull)) break;
        tc_fence_after();
        const uint32_t pa = smem_u32(sA + j * kPlaneA);
        const uint32_t pb = smem_u32(sB + j * kXPlanes * kPlaneB);
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk) {
          // 16 K rows of 128 bytes per slice; the two 64-column atoms kAtomA apart
          // B: the hi plane's MP rows followed by the mid plane's
          mma_f16(tbase, desc_mnmajor_sw128(pa + kk * 16 * 128, kAtomA),
                  desc_kmajor_sw128(pb + kk * 32), idesc, (ks > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(&bars->bfree[j]);
      }
      mma_commit(&bars->accfull);
    }
  } else {
    const int grp = (warp - 2) / kGroupWarps;
    const int t = (threadIdx.x - 64) & 127;  // thread within the group
    // x for the group's first step (in flight with the scale loads), then
    // one step ahead
    uint4 xr[kChunks];
    auto load_x = [&](int ks) {
#pragma unroll
      for (int i = 0; i < kChunks; ++i) {
        const int cid = t * kChunks + i, m = cid >> 3, kq = cid & 7;
        xr[i] = make_uint4(0u, 0u, 0u, 0u);
        if (ks < ksteps && m < M)
          xr[i] = __ldg(reinterpret_cast<const uint4*>(x + (size_t)m * K + k0 + ks * BK + kq * 8));
      }
    };
    load_x(grp);
    {
      // this tile's scale column for the K chunk, all loads in flight at
      // once; the producer and MMA warps do not wait for it
      constexpr int kPer = kMaxKc / (32 * kTransWarps);
      const int nsb = N / block;
      const float* sp = ws + (size_t)k0 * nsb + n0 / block;
      float sv[kPer];
#pragma unroll
      for (int r = 0; r < kPer; ++r) {
        const int i = (threadIdx.x - 64) + r * 32 * kTransWarps;
        sv[r] = i < kn ? __ldg(sp + (size_t)i * nsb) : 0.0f;
      }
#pragma unroll
      for (int r = 0; r < kPer; ++r) {
        const int i = (threadIdx.x - 64) + r * 32 * kTransWarps;
        if (i < kn) sS[i] = sv[r];
      }
      asm volatile("bar.sync 1, %0;" ::"n"(32 * kTransWarps) : "memory");
    }
    for (int ks = grp; ks < ksteps; ks += 2) {
      const int s = ks % STAGES, round = ks / STAGES;
      const int j = ks % kBufs, usej = ks / kBufs;
      // x' = fl(x * s) split into bf16 hi + mid, 8 values per chunk
      uint4 xh[kChunks], xm[kChunks];
#pragma unroll
      for (int i = 0; i < kChunks; ++i) {
        const int kq = (t * kChunks + i) & 7;
        const uint32_t xw[4] = {xr[i].x, xr[i].y, xr[i].z, xr[i].w};
        uint32_t hw[4], mw[4];
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          const int kk = ks * BK + kq * 8 + 2 * p;
          const float v0 = __fmul_rn(wo::bf16lo_f(xw[p]), sS[kk]);
          const float v1 = __fmul_rn(wo::bf16hi_f(xw[p]), sS[kk + 1]);
          hw[p] = wo::bf16x2_rn(v0, v1);
          mw[p] = wo::bf16x2_rn(__fsub_rn(v0, wo::bf16lo_f(hw[p])),
                                __fsub_rn(v1, wo::bf16hi_f(hw[p])));
        }
        xh[i] = make_uint4(hw[0], hw[1], hw[2], hw[3]);
        xm[i] = make_uint4(mw[0], mw[1], mw[2], mw[3]);
      }
      load_x(ks + 2);
      if (!mbar_wait_warp(&bars->full[s], round & 1, kErrTimeoutFull)) break;
      if (usej > 0 && !mbar_wait_warp(&bars->bfree[j], (usej - 1) & 1, kErrTimeoutTmemEmpty))
        break;
      // codes: 1024 units of 8 columns x 1 row per step, 8 per thread,
      // converted straight from the stage into plane j
      const uint8_t* cs = sC + s * kCodeStage;
      uint8_t* pa = sA + j * kPlaneA;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int u = t + 128 * i, k = u >> 4, c16 = u & 15;
        // MN-major, 128-byte swizzle: atom (64 columns) c16 / 8, row k, chunk c16 % 8
        const int off = (c16 >> 3) * kAtomA + k * 128 + (((c16 & 7) ^ (k & 7)) << 4);
        *reinterpret_cast<uint4*>(pa + off) = codes8_bf16<BITS>(cs + k * kCodeRow + c16 * BITS);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->empty[s]);
      uint8_t* pb = sB + j * kXPlanes * kPlaneB;
#pragma unroll
      for (int i = 0; i < kChunks; ++i) {
        const int cid = t * kChunks + i, m = cid >> 3, kq = cid & 7;
        const int off = m * 128 + ((kq ^ (m & 7)) << 4);  // K-major, 128-byte swizzle
        *reinterpret_cast<uint4*>(pb + off) = xh[i];
        *reinterpret_cast<uint4*>(pb + kPlaneB + off) = xm[i];
      }
      wo::fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->bready[j]);
    }
    // ── epilogue (group 0): TMEM (lane = column, column = token) -> out ──
    if (grp == 0 && mbar_wait_warp(&bars->accfull, 0, kErrTimeoutDone)) {
      tc_fence_after();
      const int q = warp & 3;
      const uint32_t tl = tbase + ((uint32_t)(q * 32) << 16);
      const int n = n0 + q * 32 + lane;
      float* o = out + (size_t)blockIdx.y * M * N + n;
      if (MP == 16) {
        uint32_t r[32];  // columns 0..15 hi products, 16..31 mid products
        tmem_ld32(tl, r);
        tmem_wait_ld();
#pragma unroll
        for (int m = 0; m < 16; ++m)
          if (m < M) o[(size_t)m * N] = __fadd_rn(__uint_as_float(r[m]), __uint_as_float(r[16 + m]));
      } else {
        uint32_t rh[32], rm[32];
        tmem_ld32(tl, rh);
        tmem_ld32(tl + 32, rm);
        tmem_wait_ld();
#pragma unroll
        for (int m = 0; m < 32; ++m)
          if (m < M) o[(size_t)m * N] = __fadd_rn(__uint_as_float(rh[m]), __uint_as_float(rm[m]));
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    mbar_wait(&bars->accfull, 0, kErrTimeoutDone);
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tbase, kTmemCols);
  }
}

}  // namespace dec
}  // namespace mxb
