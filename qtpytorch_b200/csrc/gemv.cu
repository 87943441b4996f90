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

// ── wide-load kernel for int4 / int8 codes ───────────────────────────────────
// KW warps share one column range and split the CTA's K slice; each lane
// loads LB bytes of codes per row (CPT columns), 8 rows ahead.  A code
// becomes an exact float with one byte permute: the offset-binary code u
// (two's complement with its sign bit flipped) placed under exponent byte
// 0x4B reads as 2^23 + u.  x * s is formed once per row and multiplied by
// the code, i.e. sum_k fl(x*s) * code instead of sum_k x * fl(code*s): the
// two differ by one fp32 rounding per term.  Warp partials are added in a
// fixed order in shared memory, so results are deterministic.
constexpr int kWideWarps = 8;

template <int BITS, int LB>
__device__ __forceinline__ void load_wide(const uint8_t* p, uint32_t (&w)[LB / 4]) {
  if constexpr (LB == 16) {
    uint4 v = __ldcs(reinterpret_cast<const uint4*>(p));
    w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
  } else if constexpr (LB == 8) {
    uint2 v = __ldcs(reinterpret_cast<const uint2*>(p));
    w[0] = v.x; w[1] = v.y;
  } else {
    w[0] = __ldcs(reinterpret_cast<const uint32_t*>(p));
  }
}

template <int BITS, int LB, int MT, typename XT, int kBatch = 4>
__global__ void __launch_bounds__(kWideWarps * 32) gemv_wide_kernel(
    const XT* __restrict__ x, int M, int K, const uint8_t* __restrict__ W,
    const float* __restrict__ ws, int N, int block, int krows, float* __restrict__ part) {
  constexpr int CPT = LB * 8 / BITS;
  constexpr int kCols = 32 * CPT;  // columns of one CTA
  // the split-reduce kernel that follows may be scheduled now (it waits
  // for this grid's completion before reading the partial sums)
  asm volatile("griddepcontrol.launch_dependents;");
  extern __shared__ __align__(16) float sm[];
  float* xs = sm;                    // [MT][krows]
  float* red = sm + MT * krows;      // [kWideWarps][MT][kCols]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int k0 = blockIdx.y * krows;
  const int kn = min(krows, K - k0);
  const int c0 = blockIdx.x * kCols + lane * CPT;
  uint64_t acc[MT][CPT / 2];  // packed pairs of columns
#pragma unroll
  for (int m = 0; m < MT; ++m)
#pragma unroll
    for (int c = 0; c < CPT / 2; ++c) acc[m][c] = 0ull;

  // The first batch of codes is requested before x is staged, so the two
  // memory round trips overlap.
  const bool live = c0 < N;
  {
    const int64_t row_bytes = (int64_t)N * BITS / 8;
    const int64_t nsb = N / block;
    const int per_warp = (kn + kWideWarps - 1) / kWideWarps;
    const int r0 = warp * per_warp, r1 = live ? min(kn, r0 + per_warp) : r0;
    const uint8_t* wp = W + (int64_t)k0 * row_bytes + (int64_t)c0 * BITS / 8;
    const float* sp = ws + (int64_t)k0 * nsb + c0 / block;
    // Two register buffers of kBatch rows: the loads of batch i+1 are in
    // flight while batch i is computed.
    uint32_t wa[kBatch][LB / 4], wb[kBatch][LB / 4];
    float sa_[kBatch], sb_[kBatch];
    auto load = [&](int rb, uint32_t (&wd)[kBatch][LB / 4], float (&sc)[kBatch]) {
#pragma unroll
      for (int b = 0; b < kBatch; ++b) {
        if (rb + b < r1) {
          load_wide<BITS, LB>(wp + (int64_t)(rb + b) * row_bytes, wd[b]);
          sc[b] = __ldg(sp + (int64_t)(rb + b) * nsb);
        } else {
#pragma unroll
          for (int q = 0; q < LB / 4; ++q) wd[b][q] = (BITS == 4) ? 0x88888888u : 0x80808080u;
          sc[b] = 0.0f;  // code 0 and scale 0: adds nothing
        }
      }
    };
    auto compute = [&](int rb, const uint32_t (&wd)[kBatch][LB / 4], const float (&sc)[kBatch]) {
#pragma unroll
      for (int b = 0; b < kBatch; ++b) {
        uint64_t code[CPT / 2];
#pragma unroll
        for (int q = 0; q < LB / 4; ++q) decode_word2<BITS>(wd[b][q], code + q * (16 / BITS));
        const int kk = min(rb + b, kn - 1);
#pragma unroll
        for (int m = 0; m < MT; ++m) {
          const float xsv = __fmul_rn(xs[m * krows + kk], sc[b]);
          const uint64_t xs2 = pack2(xsv, xsv);
#pragma unroll
          for (int c = 0; c < CPT / 2; ++c) acc[m][c] = ffma2(xs2, code[c], acc[m][c]);
        }
      }
    };
    if (r0 < r1) load(r0, wa, sa_);
    if (r0 + kBatch < r1) load(r0 + kBatch, wb, sb_);
    for (int i = threadIdx.x; i < MT * krows; i += blockDim.x) {
      const int m = i / krows, kk = i % krows;
      xs[i] = (m < M && kk < kn) ? load_as_f32(x, (int64_t)m * K + k0 + kk) : 0.0f;
    }
    __syncthreads();
    for (int rb = r0; rb < r1; rb += 2 * kBatch) {
      compute(rb, wa, sa_);
      if (rb + kBatch >= r1) break;
      if (rb + 2 * kBatch < r1) load(rb + 2 * kBatch, wa, sa_);
      compute(rb + kBatch, wb, sb_);
      if (rb + 3 * kBatch < r1) load(rb + 3 * kBatch, wb, sb_);
    }
  }
#pragma unroll
  for (int m = 0; m < MT; ++m)
#pragma unroll
    for (int c = 0; c < CPT / 2; c += 2) {
      const float2 lo = unpack2(acc[m][c]), hi = unpack2(acc[m][c + 1]);
      *reinterpret_cast<float4*>(red + (warp * MT + m) * kCols + lane * CPT + 2 * c) =
          make_float4(lo.x, lo.y, hi.x, hi.y);
    }
  __syncthreads();
  for (int i = threadIdx.x; i < MT * kCols; i += blockDim.x) {
    const int m = i / kCols, c = i % kCols;
    const int col = blockIdx.x * kCols + c;
    if (m >= M || col >= N) continue;
    float s = 0.0f;
#pragma unroll
    for (int w = 0; w < kWideWarps; ++w) s = __fadd_rn(s, red[(w * MT + m) * kCols + c]);
    part[((int64_t)blockIdx.y * M + m) * N + col] = s;
  }
}

// Launched as a programmatic dependent of the split kernel (it may start
// while that kernel drains); griddepcontrol.wait returns once the split
// kernel has completed and its partial sums are visible.
__global__ void __launch_bounds__(256) split_reduce_kernel(const float* __restrict__ part,
                                                           int splits, int64_t mn,
                                                           float* __restrict__ y) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
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

int wide_cpt(int bits, int lb) { return lb * 8 / bits; }

size_t wide_smem(int mt, int krows, int cols) {
  return (size_t)(mt * krows + kWideWarps * mt * cols) * sizeof(float);
}

template <int BITS, int LB, int MT, typename XT, int BATCH = 4>
int launch_wide_t(dim3 grid, const XT* x, int M, int K, const uint8_t* W, const float* ws, int N,
                  int block, int krows, float* part, cudaStream_t st) {
  auto kern = gemv_wide_kernel<BITS, LB, MT, XT, BATCH>;
  const size_t smem = wide_smem(MT, krows, 32 * LB * 8 / BITS);
  if (smem > 48 * 1024)
    MXB_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  kern<<<grid, kWideWarps * 32, smem, st>>>(x, M, K, W, ws, N, block, krows, part);
  MXB_LAUNCH_CHECK();
  return MXB_OK;
}

template <int BITS, typename XT>
int launch_wide(int mt, int lb, dim3 grid, const XT* x, int M, int K, const uint8_t* W,
                const float* ws, int N, int block, int krows, float* part, cudaStream_t st) {
  constexpr int LBN = BITS == 4 ? 4 : 8;  // 8 columns per thread for M > 2
  if (lb == 16) {
    if (mt == 1) return launch_wide_t<BITS, 16, 1, XT>(grid, x, M, K, W, ws, N, block, krows, part, st);
    return launch_wide_t<BITS, 16, 2, XT>(grid, x, M, K, W, ws, N, block, krows, part, st);
  }
  if (lb == 8 && mt <= 2) {
    // M = 1: 8-row batches (96 registers, two CTAs per SM) measured 10 %
    // faster than 4-row batches on configs[2]-sized int4 weights
    if (mt == 1) return launch_wide_t<BITS, 8, 1, XT, 8>(grid, x, M, K, W, ws, N, block, krows, part, st);
    return launch_wide_t<BITS, 8, 2, XT>(grid, x, M, K, W, ws, N, block, krows, part, st);
  }
  switch (mt) {
    case 4: return launch_wide_t<BITS, LBN, 4, XT>(grid, x, M, K, W, ws, N, block, krows, part, st);
    case 8: return launch_wide_t<BITS, LBN, 8, XT>(grid, x, M, K, W, ws, N, block, krows, part, st);
    default: return launch_wide_t<BITS, LBN, 16, XT>(grid, x, M, K, W, ws, N, block, krows, part, st);
  }
}

}  // namespace

namespace mxb {

GemvPlan gemv_plan(int64_t M, int64_t K, int64_t N, int bits, int kind, int block,
                   const void* w, const void* y, int x_dtype, const void* x) {
  GemvPlan p{false, 0, 0, 0};
  if (x_dtype < 0) {  // workspace query: the larger of the bf16 and fp32 plans
    GemvPlan a = gemv_plan(M, K, N, bits, kind, block, w, y, MXB_BF16, nullptr);
    GemvPlan b = gemv_plan(M, K, N, bits, kind, block, w, y, MXB_F32, nullptr);
    return a.ws_bytes >= b.ws_bytes ? a : b;
  }
  if (M >= 1 && K >= 1 && ((uintptr_t)y % 16) == 0 &&
      tc_dec_eligible(x, x_dtype, M, K, w, N, bits, kind, block)) {
    int splits, kc;
    tc_dec_plan(M, K, N, &splits, &kc);
    p.ok = true;
    p.kernel = 4;
    p.splits = splits;
    p.krows = kc;
    p.max_krows = kDecMaxKc;
    p.ws_bytes = splits > 1 ? (size_t)splits * M * N * sizeof(float) : 0;
    return p;
  }
  if (M < 1 || M > 16 || K < 1 || N < kCols) return p;
  if (N % kCols || block % kCols || N % block) return p;
  if (((uintptr_t)w % (uintptr_t)bits) || ((uintptr_t)y % 16)) return p;
  const int mt = M <= 1 ? 1 : M <= 2 ? 2 : M <= 4 ? 4 : M <= 8 ? 8 : 16;
  if (kind == MXB_KIND_INT && (bits == 4 || bits == 8)) {
    // M <= 2: int4 loads 8 bytes per lane and row (16 columns; fewer
    // registers, more resident warps), int8 16 bytes -- each measured the
    // faster of the two on configs[2]-sized weights
    const int lb = mt <= 2 ? (bits == 4 ? 8 : 16) : (bits == 4 ? 4 : 8);
    const int cpt = wide_cpt(bits, lb);
    const int cols = 32 * cpt;
    if (N % cpt == 0 && block % cpt == 0 && ((uintptr_t)w % lb) == 0) {
      // one wave: about two resident CTAs per SM, K rows a multiple of 32
      const int64_t groups = cdiv(N, cols);
      int64_t splits = (2 * kSMs) / groups;
      if (splits < 1) splits = 1;
      int64_t krows = cdiv(cdiv(K, splits), 32) * 32;
      if (krows > 1024) krows = 1024;
      splits = cdiv(K, krows);
      p.ok = true;
      p.kernel = 1;
      p.max_krows = 1024;
      p.lb = lb;
      p.splits = (int)splits;
      p.krows = (int)krows;
      p.ws_bytes = (size_t)splits * M * N * sizeof(float);
      return p;
    }
  }
  const int64_t groups = cdiv(N, kCtaCols);
  int64_t splits = cdiv(4 * kSMs, groups);
  int64_t krows = cdiv(cdiv(K, splits), 8) * 8;
  if (krows > kMaxRows) krows = kMaxRows;
  if (krows < 8) krows = 8;
  splits = cdiv(K, krows);
  p.ok = true;
  p.splits = (int)splits;
  p.krows = (int)krows;
  p.max_krows = kMaxRows;
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
  if (plan.kernel == 4) {
    if (x_dtype != MXB_BF16 || plan.krows > plan.max_krows) return MXB_E_ARG;
    rc = tc_wonly_dec(x, M, K, w, ws, N, bits, block, plan.krows, plan.splits,
                      plan.splits > 1 ? partial : y, st);
    if (rc != MXB_OK || plan.splits == 1) return rc;
  } else if (plan.kernel == 1) {
    dim3 g2((unsigned)cdiv(N, 32 * wide_cpt(bits, plan.lb)), (unsigned)plan.splits);
    if (x_dtype == MXB_F32) {
      const float* xf = static_cast<const float*>(x);
      rc = bits == 4 ? launch_wide<4>(mt, plan.lb, g2, xf, (int)M, (int)K, W, ws, (int)N, block,
                                      plan.krows, partial, st)
                     : launch_wide<8>(mt, plan.lb, g2, xf, (int)M, (int)K, W, ws, (int)N, block,
                                      plan.krows, partial, st);
    } else if (x_dtype == MXB_BF16) {
      const __nv_bfloat16* xb = static_cast<const __nv_bfloat16*>(x);
      rc = bits == 4 ? launch_wide<4>(mt, plan.lb, g2, xb, (int)M, (int)K, W, ws, (int)N, block,
                                      plan.krows, partial, st)
                     : launch_wide<8>(mt, plan.lb, g2, xb, (int)M, (int)K, W, ws, (int)N, block,
                                      plan.krows, partial, st);
    } else {
      return MXB_E_DTYPE;
    }
  } else if (x_dtype == MXB_F32)
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
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)g);
  cfg.blockDim = dim3(256);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  MXB_CUDA_TRY(cudaLaunchKernelEx(&cfg, split_reduce_kernel, (const float*)partial, plan.splits,
                                  mn, y));
  MXB_LAUNCH_CHECK();
  return MXB_OK;
}

}  // namespace mxb
