// tcgen05 packed integer GEMM for sm_100a (int8 codes, kind::i8).
//
// C = sum over K-blocks kb of fl(fl(P_kb * sa[m, kb]) * sb[kb, n]), in kb
// order, P_kb the exact int32 product of one 128-wide K-block
// (mxtorch.py:1299-1385).  One CTA owns a 128x128 tile of C:
//   warp 0      TMA producer: A [128 x 128 B] (K-major) and B [128 K x 128 N]
//               (N-major, B's native row-major layout) per K-block, 128-byte
//               swizzle, STAGES-deep ring of shared-memory stages;
//   warp 1      allocates 256 TMEM columns and issues 4 x tcgen05.mma
//               (M=128, N=128, K=32, s8 x s8 -> s32) per K-block into one of
//               two TMEM accumulators, so the MMAs of K-block kb+1 overlap
//               the promotion of kb;
//   warps 2..17 promotion: tcgen05.ld the int32 tile (one TMEM lane = one
//               row, 32 columns per warp), convert exactly (I2F), apply both
//               scales and add into fp32 registers (packed f32x2 ops), one rounding per
//               step.  The fp32 accumulator is bit-identical to the
//               reference's.
// Sub-byte codes (int4 / int2 / int1) are first widened to int8 in the
// workspace.  All waits are bounded (tc_ptx.cuh).
#include "mxb_common.cuh"
#include "mxb_internal.h"

#include <cuda.h>
#include <cstring>

namespace mxb {
__device__ int g_mxb_device_error = 0;
}

#include "tc_ptx.cuh"
#include "wonly_tc.cuh"
#include "wonly_dec.cuh"

namespace mxb {

namespace {

constexpr int BM = 128, BN = 128, BKB = 128;  // tile rows, cols, K-block bytes
constexpr int STAGES = 4;
constexpr int kEpiWarps = 16;
constexpr int kEpiCols = BN * 4 / kEpiWarps;  // columns per epilogue warp (32)
static_assert(kEpiCols == 32, "one tcgen05.ld x32 per warp and K-block");
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr int kTileA = BM * BKB;   // 16 KB
constexpr int kTileB = BN * BKB;   // 16 KB
constexpr int kTmemCols = 2 * BN;  // two int32 accumulators
constexpr size_t kBarsBytes = 8192;  // >= sizeof(Bars), checked below
constexpr size_t kSmemBytes = 1024 + (size_t)STAGES * (kTileA + kTileB) + kBarsBytes;
// int16d codes of a tile staged in the TMA ring (idle once the last MMA is
// done) as two boxes of 128 rows x 128 bytes (64 codes) in the 128-byte
// swizzled layout the output tensor maps use (16-byte chunk c of row r at
// chunk c ^ (r & 7): the lanes' 16-byte writes of consecutive rows hit
// different bank groups)
constexpr int kStgBox = BM * 128;
static_assert(2 * kStgBox <= STAGES * kTileA, "staging fits the A ring");

// Tensor maps of the int16d outputs (codes as 32-bit words, [M][N_full / 2],
// box 32 words x 128 rows, 128-byte swizzle), one per QOut output.
struct OutMaps {
  CUtensorMap m[kMaxPeers];
};

struct Bars {
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint64_t done;
  uint32_t tmem_base;
  // per-warp double buffer of B scales, read back as float4 broadcasts
  alignas(16) float sbw[kEpiWarps][2 * kEpiCols];
  // per-row absmax of each 32-column slice, for the fused requantization
  float slice_amax[BN / kEpiCols][BM];
  float row_scale[BM];  // the tile rows' int16d scales, staged for the copy-out
};
static_assert(sizeof(Bars) <= kBarsBytes, "barrier block overflows its shared-memory slot");
static_assert(offsetof(Bars, sbw) % 16 == 0, "float4 reads of sbw need 16-byte alignment");

// Cross-rank completion barrier, launched right after a rank's sharded
// matmul on the same stream (so every store of that kernel, over NVLink
// included, is complete when it runs): one thread raises this rank's call
// counter, signals it to every rank with a system-scope release store into
// their barrier blocks and waits, bounded by kWaitLimitNs, until every rank
// has signalled the same call.  The counters advance in step on every rank
// (one per call) and live on the device, so the protocol needs no host
// state and replays under a CUDA graph.  A wait that gives up records
// kErrTimeoutPeer.
__global__ void __launch_bounds__(32) cross_rank_barrier_kernel(const __grid_constant__ QOut q) {
  if (threadIdx.x != 0) return;
  unsigned long long* mine = q.sync[q.rank];
  __threadfence_system();
  const unsigned long long call = mine[1] + 1;
  mine[1] = call;
  for (int r = 0; r < q.count; ++r) {
    unsigned long long* dst = q.sync[r] + 8 + q.rank;
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(dst), "l"(call) : "memory");
  }
  const uint64_t t0 = globaltimer_ns();
  for (int r = 0; r < q.count; ++r) {
    const unsigned long long* src = mine + 8 + r;
    for (uint32_t i = 0;; ++i) {
      unsigned long long v;
      asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(src) : "memory");
      if (v >= call) break;
      if ((i & 63) == 63 && globaltimer_ns() - t0 > kWaitLimitNs) {
        atomicCAS(&g_mxb_device_error, 0, kErrTimeoutPeer);
        return;
      }
      __nanosleep(64);
    }
  }
}

// B_KMAJOR: B is given as B^T [N, K] (each column's K run contiguous: the
// layout of a matrix quantized along K) and read as a K-major operand.
template <bool B_KMAJOR>
__global__ void __launch_bounds__(kThreads, 1)
    qgemm_tc_kernel(const __grid_constant__ CUtensorMap tmap_a,
                    const __grid_constant__ CUtensorMap tmap_b, const float* __restrict__ sa,
                    const float* __restrict__ sb, int M, int N, int K, float* __restrict__ C,
                    const __grid_constant__ QOut qout, const __grid_constant__ OutMaps omaps) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * kTileA;
  Bars* bars = reinterpret_cast<Bars*>(sB + STAGES * kTileB);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  const int kbn = K / BKB;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars->tfull[b], 1);
      mbar_init(&bars->tempty[b], kEpiWarps);
    }
    mbar_init(&bars->done, 1);
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmap_a);
    prefetch_tmap(&tmap_b);
  }
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
      for (int kb = 0; kb < kbn; ++kb) {
        const int s = kb % STAGES, round = kb / STAGES;
        if (round > 0 && !mbar_wait(&bars->empty[s], (round - 1) & 1, kErrTimeoutEmpty)) break;
        mbar_expect_tx(&bars->full[s], kTileA + kTileB);
        tma_load_2d(sA + s * kTileA, &tmap_a, &bars->full[s], kb * BKB, m0);
        if (B_KMAJOR)
          tma_load_2d(sB + s * kTileB, &tmap_b, &bars->full[s], kb * BKB, n0);
        else
          tma_load_2d(sB + s * kTileB, &tmap_b, &bars->full[s], n0, kb * BKB);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc =
          make_idesc(/*S32*/ 2, /*s8*/ 1, 0, /*B N-major*/ B_KMAJOR ? 0 : 1, BM, BN);
      for (int kb = 0; kb < kbn; ++kb) {
        const int s = kb % STAGES, round = kb / STAGES;
        const int b = kb & 1, use = kb >> 1;
        if (!mbar_wait(&bars->full[s], round & 1, kErrTimeoutFull)) break;
        if (use > 0 && !mbar_wait(&bars->tempty[b], (use - 1) & 1, kErrTimeoutTmemEmpty)) break;
        tc_fence_after();
        const uint32_t a0 = smem_u32(sA + s * kTileA), b0 = smem_u32(sB + s * kTileB);
#pragma unroll
        for (int kk = 0; kk < BKB / 32; ++kk) {
          const uint64_t bd = B_KMAJOR ? desc_kmajor_sw128(b0 + kk * 32)
                                       : desc_mnmajor_sw128(b0 + kk * 32 * BN, kTileB);
          mma_i8(tbase + b * BN, desc_kmajor_sw128(a0 + kk * 32), bd, idesc, kk > 0 ? 1u : 0u);
        }
        mma_commit(&bars->empty[s]);
        mma_commit(&bars->tfull[b]);
      }
      mma_commit(&bars->done);
    }
  } else {
    const int ew = warp - 2;
    const int q = warp & 3;                 // TMEM lane quadrant this warp may access
    const int col0 = (ew >> 2) * kEpiCols;  // this warp's column slice
    const int row = q * 32 + lane;
    const int m = m0 + row;
    // fp32 accumulator as packed pairs (f32x2 ops round each lane like the
    // scalar op, so results stay bit-identical); measured faster than one
    // register per column with scalar adds (0.192 vs 0.203 ms at 4096^3)
    uint64_t acc[kEpiCols / 2];
#pragma unroll
    for (int c = 0; c < kEpiCols / 2; ++c) acc[c] = 0ull;
    // Scales are fetched one K-block ahead: sa (one per row) into a register,
    // this warp's sb slice one value per lane, staged through a per-warp
    // double buffer in shared memory and read back as broadcasts.
    float* sbw = bars->sbw[ew];
    const float* sap = sa + (size_t)m * kbn;
    const float* sbrow = sb + n0 + col0 + lane;
    float sa_next = __ldg(sap);
    float sb_next = __ldg(sbrow);
    for (int kb = 0; kb < kbn; ++kb) {
      const int b = kb & 1, use = kb >> 1;
      const float sa_v = sa_next;
      sbw[b * kEpiCols + lane] = sb_next;
      __syncwarp();
      if (kb + 1 < kbn) {
        sa_next = __ldg(sap + kb + 1);
        sb_next = __ldg(sbrow + (size_t)(kb + 1) * N);
      }
      if (!mbar_wait_warp(&bars->tfull[b], use & 1, kErrTimeoutTmemFull)) break;
      tc_fence_after();
      uint32_t r[kEpiCols];
      const uint32_t taddr = tbase + ((uint32_t)(q * 32) << 16) + b * BN + col0;
      tmem_ld32(taddr, r);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->tempty[b]);
      const uint64_t sa2 = pack2(sa_v, sa_v);
      const ulonglong2* sbp = reinterpret_cast<const ulonglong2*>(sbw + b * kEpiCols);
#pragma unroll
      for (int c4 = 0; c4 < kEpiCols / 4; ++c4) {
        const ulonglong2 s4 = sbp[c4];
        const uint64_t sv[2] = {s4.x, s4.y};
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int c = c4 * 4 + 2 * j;
          // int -> fp32 is exact (|P| <= 128 * 128^2 < 2^24); the conversion
          // runs outside the FMA pipe, which the three FP32 operations keep busy
          const uint64_t pf = pack2(__int2float_rn((int)r[c]), __int2float_rn((int)r[c + 1]));
          // products packed; the add stays scalar so it is never fused
          // with the multiply (a fused add would skip one rounding)
          const float2 t = unpack2(fmul2(fmul2(pf, sa2), sv[j]));
          const float2 a = unpack2(acc[c / 2]);
          acc[c / 2] = pack2(__fadd_rn(a.x, t.x), __fadd_rn(a.y, t.y));
        }
      }
    }
    if (C != nullptr) {
      float4* out = reinterpret_cast<float4*>(C + (size_t)m * N + n0 + col0);
#pragma unroll
      for (int c4 = 0; c4 < kEpiCols / 4; ++c4) {
        const float2 lo = unpack2(acc[2 * c4]), hi = unpack2(acc[2 * c4 + 1]);
        out[c4] = make_float4(lo.x, lo.y, hi.x, hi.y);
      }
    }
    if (qout.count > 0) {
      // Fused int16d requantization (mxtorch.py:1371-1378): the 128 columns
      // of this tile row are one scale block (N % 128 == 0, block 128).
      float a = 0.0f;
#pragma unroll
      for (int c = 0; c < kEpiCols / 2; ++c) {
        const float2 v = unpack2(acc[c]);
        a = amax_step(amax_step(a, v.x), v.y);
      }
      bars->slice_amax[ew >> 2][row] = a;
      asm volatile("bar.sync 1, %0;" ::"n"(kEpiWarps * 32) : "memory");  // promotion warps only
#pragma unroll
      for (int s = 0; s < BN / kEpiCols; ++s) a = nan_max(a, bars->slice_amax[s][row]);
      const float cs = __fdiv_rn(a < 1e-12f ? 1e-12f : a, 32767.0f);
      uint32_t w[kEpiCols / 2];
#pragma unroll
      for (int c = 0; c < kEpiCols / 2; ++c) {
        const float2 v = unpack2(acc[c]);
        uint32_t code[2];
        const float vv[2] = {v.x, v.y};
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const float qv = nan_min(nan_max(__fdiv_rn(vv[h], cs), -32767.0f), 32767.0f);
          // round half to even by adding 1.5 * 2^23; NaN stores code 0
          const uint32_t bits = __float_as_uint(__fadd_rn(qv, 12582912.0f)) & 0xFFFFu;
          code[h] = qv == qv ? bits : 0u;
        }
        w[c] = code[0] | (code[1] << 16);
      }
      // Stage the tile's codes in shared memory, then one thread stores both
      // boxes with TMA tile stores into every output of the list: this
      // rank's, or, for a column-sharded matmul, the full-width output of
      // every rank (peer memory over NVLink) at this shard's column offset.
      // Two 16 KB stores per output keep NVLink packets full and leave the
      // threads free; the CTA waits only until the staging has been read.
      uint8_t* stg = sA + (col0 >> 6) * kStgBox + row * 128;
      const int ch0 = (col0 & 63) >> 3;  // first 16-byte chunk of this warp's columns
#pragma unroll
      for (int c = 0; c < kEpiCols / 8; ++c)
        *reinterpret_cast<uint4*>(stg + (((ch0 + c) ^ (row & 7)) << 4)) =
            make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
      if (ew < 4) bars->row_scale[row] = cs;
      fence_proxy_async_shared();
      asm volatile("bar.sync 2, %0;" ::"n"(kEpiWarps * 32) : "memory");
      const int te = threadIdx.x - 64;  // 0 .. 511
      if (te == 0) {
        const int x0 = (qout.col_off + n0) >> 1;  // in 32-bit words: a multiple of 64
        for (int r = 0; r < qout.count; ++r) {
          tma_store_2d(&omaps.m[r], sA, x0, m0);
          tma_store_2d(&omaps.m[r], sA + kStgBox, x0 + 32, m0);
        }
        bulk_commit();
      }
      if (te < BM) {
        const size_t e = (size_t)(m0 + te) * qout.row_stride + qout.col_off + n0;
        for (int r = 0; r < qout.count; ++r) qout.scales[r][e / BN] = bars->row_scale[te];
      }
      // The row copies (over NVLink for peers) finish while the next tiles
      // compute, and are complete when the kernel is, which the post-launch
      // barrier (the cross-rank barrier kernel, or a collective) orders
      // before any rank reads.
      if (te == 0) bulk_wait_read();
    }
  }
  __syncthreads();
  if (warp == 1) {
    mbar_wait(&bars->done, 0, kErrTimeoutDone);
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tbase, kTmemCols);
  }
}

// Integer value of a raw code.  The reference's matmul sign-extends every
// width, so a 1-bit code is 0 or -1 there; `pm1` gives 1-bit codes their
// dequantized meaning instead (raw 0 -> +1, raw 1 -> -1), for the k-major
// matmul whose result is the quantized product.
template <int BITS>
__device__ __forceinline__ int8_t code_value(uint32_t raw, bool pm1) {
  if (BITS == 1 && pm1) return (raw & 1u) ? (int8_t)-1 : (int8_t)1;
  return (int8_t)sext(raw, BITS);
}

// Scales of a matrix quantized along K (B^T [N, K], K % block == 0:
// s[n, kb]) -> the [K/block, N] layout the GEMM kernels read.
__global__ void __launch_bounds__(256) transpose_scales_kernel(const float* __restrict__ s,
                                                               int kbn, int N,
                                                               float* __restrict__ out) {
  const int64_t total = (int64_t)kbn * N;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t kb = i / N, n = i % N;
    out[i] = s[n * kbn + kb];
  }
}

// B^T [N, K] packed codes -> B [K, N] one signed byte per code (for the
// CUDA-core kernel, which reads B row-major).
template <int BITS>
__global__ void __launch_bounds__(256) widen_transpose_kernel(const uint8_t* __restrict__ bt,
                                                              int K, int N, bool pm1,
                                                              int8_t* __restrict__ out) {
  constexpr int PER = 8 / BITS;
  const int64_t total = (int64_t)K * N;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t k = i / N, n = i % N, e = n * K + k;
    const uint32_t raw = (bt[e / PER] >> ((e % PER) * BITS)) & ((1u << BITS) - 1u);
    out[i] = code_value<BITS>(raw, pm1);
  }
}

// Widen packed sub-byte codes to one signed byte per code.
template <int BITS>
__global__ void __launch_bounds__(256) widen_codes_kernel(const uint8_t* __restrict__ p,
                                                          int64_t n, bool pm1,
                                                          int8_t* __restrict__ out) {
  constexpr int PER = 8 / BITS;
  const int64_t nbytes = (n + PER - 1) / PER;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nbytes;
       i += (int64_t)gridDim.x * blockDim.x) {
    const uint32_t b = p[i];
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const int64_t e = i * PER + j;
      if (e < n) out[e] = code_value<BITS>((b >> (j * BITS)) & ((1u << BITS) - 1u), pm1);
    }
  }
}

}  // namespace

int transpose_scales(const float* s, int64_t kbn, int64_t N, float* out, cudaStream_t st) {
  int64_t g = cdiv(kbn * N, 256);
  if (g > kSMs * 8) g = kSMs * 8;
  transpose_scales_kernel<<<(unsigned)g, 256, 0, st>>>(s, (int)kbn, (int)N, out);
  MXB_LAUNCH_CHECK();
  return MXB_OK;
}

int widen_transpose(const void* bt, int64_t K, int64_t N, int bits, bool pm1, int8_t* out,
                    cudaStream_t st) {
  int64_t g = cdiv(K * N, 256);
  if (g > kSMs * 16) g = kSMs * 16;
  const uint8_t* p = static_cast<const uint8_t*>(bt);
  switch (bits) {
    case 1: widen_transpose_kernel<1><<<(unsigned)g, 256, 0, st>>>(p, (int)K, (int)N, pm1, out); break;
    case 2: widen_transpose_kernel<2><<<(unsigned)g, 256, 0, st>>>(p, (int)K, (int)N, pm1, out); break;
    case 4: widen_transpose_kernel<4><<<(unsigned)g, 256, 0, st>>>(p, (int)K, (int)N, pm1, out); break;
    case 8: widen_transpose_kernel<8><<<(unsigned)g, 256, 0, st>>>(p, (int)K, (int)N, pm1, out); break;
    default: return MXB_E_DTYPE;
  }
  MXB_LAUNCH_CHECK();
  return MXB_OK;
}

namespace {

int widen(const void* p, int64_t n, int bits, int8_t* out, cudaStream_t st, bool pm1 = false) {
  const int per = 8 / bits;
  int64_t g = cdiv(cdiv(n, per), 256);
  if (g > kSMs * 16) g = kSMs * 16;
  const uint8_t* src = static_cast<const uint8_t*>(p);
  switch (bits) {
    case 1: widen_codes_kernel<1><<<(unsigned)g, 256, 0, st>>>(src, n, pm1, out); break;
    case 2: widen_codes_kernel<2><<<(unsigned)g, 256, 0, st>>>(src, n, pm1, out); break;
    case 4: widen_codes_kernel<4><<<(unsigned)g, 256, 0, st>>>(src, n, pm1, out); break;
    default: return MXB_E_DTYPE;
  }
  MXB_LAUNCH_CHECK();
  return MXB_OK;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda link).
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

}  // namespace

int widen_codes(const void* p, int64_t n, int bits, int8_t* out, bool pm1, cudaStream_t st) {
  return widen(p, n, bits, out, st, pm1);
}


// 2-D row-major byte matrix [rows][cols] -> tensor map with a 128x128-byte box,
// 128-byte swizzle.
// 2-D row-major matrix [rows][cols] of `esize`-byte elements -> tensor map.
int make_tmap_2d(CUtensorMap* map, CUtensorMapDataType dt, uint32_t esize, const void* base,
                 uint64_t cols, uint64_t rows, uint32_t box_cols, uint32_t box_rows,
                 CUtensorMapSwizzle swz) {
  EncodeTiledFn enc = encode_fn();
  if (enc == nullptr) return MXB_E_CUDA;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * esize};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t elem[2] = {1, 1};
  CUresult r = enc(map, dt, 2, const_cast<void*>(base), dims, strides, box, elem,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? MXB_OK : MXB_E_CUDA;
}

int make_tmap_u8(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows,
                 uint32_t box_cols, uint32_t box_rows) {
  return make_tmap_2d(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, base, cols, rows, box_cols, box_rows,
                      CU_TENSOR_MAP_SWIZZLE_128B);
}

bool tc_qgemm_eligible(int64_t M, int64_t K, int64_t N, int bits, int block, bool sa_ok,
                       bool sb_ok, const void* a, const void* b, const float* c) {
  if (block != BKB || !sa_ok || !sb_ok) return false;
  if (bits != 8 && bits != 4 && bits != 2 && bits != 1) return false;
  if (M % BM || N % BN || K % BKB || M <= 0 || N <= 0 || K <= 0) return false;
  if (bits == 8 && (((uintptr_t)a | (uintptr_t)b) & 15)) return false;
  if ((uintptr_t)c & 15) return false;
  return true;
}

size_t tc_qgemm_workspace(int64_t M, int64_t K, int64_t N, int bits) {
  if (bits == 8) return 0;
  return (size_t)((M * K + 255) / 256 * 256 + (K * N + 255) / 256 * 256);
}

int tc_qgemm(const void* a, const float* sa, const void* b, const float* sb, int64_t M,
             int64_t K, int64_t N, int bits, int block, float* C, const QOut* qout, void* ws,
             size_t wsb, bool b_kmajor, cudaStream_t st) {
  (void)block;
  const void* a8 = a;
  const void* b8 = b;
  if (bits != 8) {
    if (wsb < tc_qgemm_workspace(M, K, N, bits)) return MXB_E_WORKSPACE;
    int8_t* wa = static_cast<int8_t*>(ws);
    int8_t* wb = wa + (M * K + 255) / 256 * 256;
    int rc = widen(a, M * K, bits, wa, st, b_kmajor);
    if (rc != MXB_OK) return rc;
    rc = widen(b, K * N, bits, wb, st, b_kmajor);
    if (rc != MXB_OK) return rc;
    a8 = wa;
    b8 = wb;
  }
  CUtensorMap ta, tb;
  if (make_tmap_u8(&ta, a8, (uint64_t)K, (uint64_t)M, BKB, BM) != MXB_OK) return MXB_E_CUDA;
  if (b_kmajor ? make_tmap_u8(&tb, b8, (uint64_t)K, (uint64_t)N, BKB, BN)
               : make_tmap_u8(&tb, b8, (uint64_t)N, (uint64_t)K, BN, BKB)) {
    return MXB_E_CUDA;
  }
  auto kern = b_kmajor ? qgemm_tc_kernel<true> : qgemm_tc_kernel<false>;
  // set per call: the attribute belongs to the current device's context
  MXB_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)kSmemBytes));
  dim3 grid((unsigned)(N / BN), (unsigned)(M / BM));
  QOut none{};
  OutMaps om;
  memset(&om, 0, sizeof(om));
  if (qout) {
    for (int r = 0; r < qout->count; ++r)
      if (make_tmap_2d(&om.m[r], CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, qout->words[r],
                       (uint64_t)qout->row_stride / 2, (uint64_t)M, 32, BM,
                       CU_TENSOR_MAP_SWIZZLE_128B) != MXB_OK)
        return MXB_E_CUDA;
  }
  kern<<<grid, kThreads, kSmemBytes, st>>>(ta, tb, sa, sb, (int)M, (int)N, (int)K, C,
                                           qout ? *qout : none, om);
  MXB_LAUNCH_CHECK();
  if (qout && qout->sync[0] != nullptr) {
    cross_rank_barrier_kernel<<<1, 32, 0, st>>>(*qout);
    MXB_LAUNCH_CHECK();
  }
  return MXB_OK;
}

int peer_barrier(unsigned long long* const* sync, int nranks, int rank, cudaStream_t st) {
  QOut q{};
  q.count = nranks;
  q.rank = rank;
  for (int r = 0; r < nranks; ++r) q.sync[r] = sync[r];
  cross_rank_barrier_kernel<<<1, 32, 0, st>>>(q);
  MXB_LAUNCH_CHECK();
  return MXB_OK;
}

// ── weight-only GEMM (wonly_tc.cuh) ──────────────────────────────────────────
bool tc_wonly_eligible(const void* x, int x_dtype, int64_t M, int64_t K, const void* w,
                       int64_t N, int bits, int kind, int block, const float* y, bool kmajor) {
  if (x_dtype != MXB_BF16 || M <= 16) return false;
  if (K % wo::BK || N % wo::BN || block % 8) return false;
  if (kind == MXB_KIND_FLOAT ? bits != 4 : !(bits == 1 || bits == 2 || bits == 4 || bits == 8))
    return false;
  if (kmajor) {
    // the K-major code box is BK * bits / 8 bytes wide: at least 16
    if (bits < 2 || K % block) return false;
  } else if (N % block) {
    return false;
  }
  if (((uintptr_t)x | (uintptr_t)w | (uintptr_t)y) & 15) return false;
  return true;
}

template <int BITS, int KIND, bool FAST, bool KMAJ>
static int wonly_launch(const CUtensorMap& tx, const CUtensorMap& tw, const float* ws, int M,
                        int N, int K, int block, float* y, cudaStream_t st) {
  auto kern = wo::wonly_tc_kernel<BITS, KIND, FAST, KMAJ>;
  MXB_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)wo::kSmemBytes));
  dim3 grid((unsigned)(N / wo::BN), (unsigned)cdiv(M, wo::BM));
  kern<<<grid, wo::kThreads, wo::kSmemBytes, st>>>(tx, tw, ws, M, N, K, block, y);
  MXB_LAUNCH_CHECK();
  return MXB_OK;
}

template <int BITS, int KIND>
static int wonly_mode(bool fast, bool kmajor, const CUtensorMap& tx, const CUtensorMap& tw,
                      const float* ws, int M, int N, int K, int block, float* y,
                      cudaStream_t st) {
  if (kmajor) {
    if constexpr (BITS >= 2)
      return fast ? wonly_launch<BITS, KIND, true, true>(tx, tw, ws, M, N, K, block, y, st)
                  : wonly_launch<BITS, KIND, false, true>(tx, tw, ws, M, N, K, block, y, st);
    return MXB_E_DTYPE;
  }
  return fast ? wonly_launch<BITS, KIND, true, false>(tx, tw, ws, M, N, K, block, y, st)
              : wonly_launch<BITS, KIND, false, false>(tx, tw, ws, M, N, K, block, y, st);
}

int tc_wonly(const void* x, int64_t M, int64_t K, const void* w, const float* ws, int64_t N,
             int bits, int kind, int block, int mode, float* y, cudaStream_t st, bool kmajor) {
  CUtensorMap tx, tw;
  if (make_tmap_2d(&tx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, x, (uint64_t)K, (uint64_t)M, wo::BK,
                   128, CU_TENSOR_MAP_SWIZZLE_128B) != MXB_OK)
    return MXB_E_CUDA;
  if (kmajor) {
    const uint64_t row_bytes = (uint64_t)K * bits / 8;  // one N row of W [N, K]
    if (make_tmap_2d(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, w, row_bytes, (uint64_t)N,
                     (uint32_t)(wo::BK * bits / 8), wo::BN, CU_TENSOR_MAP_SWIZZLE_NONE) != MXB_OK)
      return MXB_E_CUDA;
  } else {
    const uint64_t row_bytes = (uint64_t)N * bits / 8;
    if (make_tmap_2d(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, w, row_bytes, (uint64_t)K,
                     (uint32_t)(wo::BN * bits / 8), wo::BK, CU_TENSOR_MAP_SWIZZLE_NONE) != MXB_OK)
      return MXB_E_CUDA;
  }
  const bool fast = mode == MXB_MODE_FAST;
  const int iM = (int)M, iN = (int)N, iK = (int)K;
  if (kind == MXB_KIND_FLOAT)
    return wonly_mode<4, MXB_KIND_FLOAT>(fast, kmajor, tx, tw, ws, iM, iN, iK, block, y, st);
  switch (bits) {
    case 1: return wonly_mode<1, MXB_KIND_INT>(fast, kmajor, tx, tw, ws, iM, iN, iK, block, y, st);
    case 2: return wonly_mode<2, MXB_KIND_INT>(fast, kmajor, tx, tw, ws, iM, iN, iK, block, y, st);
    case 4: return wonly_mode<4, MXB_KIND_INT>(fast, kmajor, tx, tw, ws, iM, iN, iK, block, y, st);
    case 8: return wonly_mode<8, MXB_KIND_INT>(fast, kmajor, tx, tw, ws, iM, iN, iK, block, y, st);
  }
  return MXB_E_DTYPE;
}

// ── decode-regime weight-only linear (wonly_dec.cuh) ─────────────────────────
bool tc_dec_eligible(const void* x, int x_dtype, int64_t M, int64_t K, const void* w, int64_t N,
                     int bits, int kind, int block) {
  if (x_dtype != MXB_BF16 || kind != MXB_KIND_INT) return false;
  if (!(bits == 1 || bits == 2 || bits == 4 || bits == 8)) return false;
  // M <= 2 stays on the CUDA-core GEMV, which streams the weight faster when
  // there is at most two rows of work per code
  if (M < 3 || M > 32 || K % dec::BK || N % dec::BN || block % dec::BN || N % block) return false;
  if (((uintptr_t)x | (uintptr_t)w) & 15) return false;
  return true;
}

void tc_dec_plan(int64_t M, int64_t K, int64_t N, int* splits, int* kc) {
  // one wave of 128-column groups x K splits: three CTAs per SM for M <= 16
  // (about 72 KB of shared memory each; measured 10 % faster than two at
  // 16 x 4096 x 11008), two for 32 padded token rows (larger x planes)
  const int64_t groups = N / dec::BN, steps = K / dec::BK;
  int64_t sp = ((M <= 16 ? 3 : 2) * kSMs) / groups;
  if (sp < 1) sp = 1;
  if (sp > steps) sp = steps;
  int64_t c = cdiv(steps, sp) * dec::BK;
  if (c > dec::kMaxKc) c = dec::kMaxKc;
  *kc = (int)c;
  *splits = (int)cdiv(K, c);
}

template <int BITS, int MP>
static int dec_launch(const CUtensorMap& tw, const __nv_bfloat16* x, const float* ws, int M,
                      int N, int K, int block, int kc, int splits, float* out, cudaStream_t st) {
  auto kern = dec::wonly_dec_kernel<BITS, MP>;
  const size_t smem = dec::smem_bytes<BITS, MP>(kc);
  MXB_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  dim3 grid((unsigned)(N / dec::BN), (unsigned)splits);
  kern<<<grid, dec::kThreads, smem, st>>>(tw, x, ws, M, N, K, block, kc, out);
  MXB_LAUNCH_CHECK();
  return MXB_OK;
}

template <int BITS>
static int dec_mp(const CUtensorMap& tw, const __nv_bfloat16* x, const float* ws, int M, int N,
                  int K, int block, int kc, int splits, float* out, cudaStream_t st) {
  return M <= 16 ? dec_launch<BITS, 16>(tw, x, ws, M, N, K, block, kc, splits, out, st)
                 : dec_launch<BITS, 32>(tw, x, ws, M, N, K, block, kc, splits, out, st);
}

int tc_wonly_dec(const void* x, int64_t M, int64_t K, const void* w, const float* ws, int64_t N,
                 int bits, int block, int kc, int splits, float* out, cudaStream_t st) {
  if (kc <= 0 || kc % dec::BK || kc > dec::kMaxKc || (int64_t)splits * kc < K) return MXB_E_ARG;
  CUtensorMap tw;
  const uint64_t row_bytes = (uint64_t)N * bits / 8;
  if (make_tmap_2d(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, w, row_bytes, (uint64_t)K,
                   (uint32_t)(dec::BN * bits / 8), dec::BK, CU_TENSOR_MAP_SWIZZLE_NONE) != MXB_OK)
    return MXB_E_CUDA;
  const __nv_bfloat16* xb = static_cast<const __nv_bfloat16*>(x);
  const int iM = (int)M, iN = (int)N, iK = (int)K;
  switch (bits) {
    case 1: return dec_mp<1>(tw, xb, ws, iM, iN, iK, block, kc, splits, out, st);
    case 2: return dec_mp<2>(tw, xb, ws, iM, iN, iK, block, kc, splits, out, st);
    case 4: return dec_mp<4>(tw, xb, ws, iM, iN, iK, block, kc, splits, out, st);
    case 8: return dec_mp<8>(tw, xb, ws, iM, iN, iK, block, kc, splits, out, st);
  }
  return MXB_E_DTYPE;
}

}  // namespace mxb

namespace mxb {
// Device address of the error word for kernels of other translation units
// (looked up with the device current; nullptr if that fails).
int* device_error_ptr() {
  void* p = nullptr;
  return cudaGetSymbolAddress(&p, g_mxb_device_error) == cudaSuccess ? static_cast<int*>(p)
                                                                    : nullptr;
}
}  // namespace mxb

extern "C" int mxb_device_error(int clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, mxb::g_mxb_device_error, sizeof(int)) != cudaSuccess)
    return MXB_E_CUDA;
  if (clear && v != 0) {
    int z = 0;
    if (cudaMemcpyToSymbol(mxb::g_mxb_device_error, &z, sizeof(int)) != cudaSuccess)
      return MXB_E_CUDA;
  }
  return v;
}
