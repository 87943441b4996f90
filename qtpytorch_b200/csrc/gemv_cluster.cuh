// Cluster GEMV for int4 / int8 codes, M <= 2 (the decode case of configs[2]).
// Included by gemv.cu inside its anonymous namespace.
//
// The 8 K-slices of one 512-column group run as one thread-block cluster
// (cluster dims 1 x 8).  Each CTA streams its slice of W^T with 8-byte loads
// per lane (a warp reads 256 contiguous bytes of a row), two batches of 8
// rows in flight per thread, decodes codes exactly (byte permute under
// exponent 0x4B) and accumulates fl(x*s) * code with packed f32x2 FMA.  Warp
// partials are added in shared memory; then, after a cluster barrier, CTA
// rank r adds the 8 CTAs' partials for columns [64r, 64r + 64) through
// distributed shared memory, in rank order, and writes y.  No partial-sum
// workspace and no second kernel; the result is deterministic.

constexpr int kClWarps = 8;
constexpr int kClSplits = 8;   // cluster size along K
constexpr int kClLB = 8;       // code bytes per lane and row
constexpr int kClBatch = 8;    // rows per load batch

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Read a float from the same shared-memory offset in CTA `rank` of the cluster.
__device__ __forceinline__ float ld_cluster_f32(const float* local, uint32_t rank) {
  uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(local)), ra;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(a), "r"(rank));
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(ra) : "memory");
  return v;
}

template <int BITS, int MT, typename XT>
__global__ void __launch_bounds__(kClWarps * 32) gemv_cluster_kernel(
    const XT* __restrict__ x, int M, int K, const uint8_t* __restrict__ W,
    const float* __restrict__ ws, int N, int block, int krows, float* __restrict__ y) {
  constexpr int CPT = kClLB * 8 / BITS;  // columns per lane
  constexpr int kCols = 32 * CPT;        // columns of one CTA
  extern __shared__ __align__(16) float sm[];
  float* xs = sm;                                // [MT][krows]
  float* red = sm + MT * krows;                  // [kClWarps][MT][kCols]
  float* cta_part = red + kClWarps * MT * kCols; // [MT][kCols]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int k0 = blockIdx.y * krows;
  const int kn = max(0, min(krows, K - k0));
  for (int i = threadIdx.x; i < MT * krows; i += blockDim.x) {
    const int m = i / krows, kk = i % krows;
    xs[i] = (m < M && kk < kn) ? load_as_f32(x, (int64_t)m * K + k0 + kk) : 0.0f;
  }
  __syncthreads();

  const int c_cta = blockIdx.x * kCols;
  const int c0 = c_cta + lane * CPT;
  uint64_t acc[MT][CPT / 2];
#pragma unroll
  for (int m = 0; m < MT; ++m)
#pragma unroll
    for (int c = 0; c < CPT / 2; ++c) acc[m][c] = 0ull;

  if (c0 < N && kn > 0) {
    const int64_t row_bytes = (int64_t)N * BITS / 8;
    const int64_t nsb = N / block;
    const int per_warp = (kn + kClWarps - 1) / kClWarps;
    const int r0 = warp * per_warp, r1 = min(kn, r0 + per_warp);
    const uint8_t* wp = W + (int64_t)k0 * row_bytes + (int64_t)c0 * BITS / 8;
    const float* sp = ws + (int64_t)k0 * nsb + c0 / block;
    uint2 wa[kClBatch], wb[kClBatch];
    float sa_[kClBatch], sb_[kClBatch];
    auto load = [&](int rb, uint2 (&wd)[kClBatch], float (&sc)[kClBatch]) {
#pragma unroll
      for (int b = 0; b < kClBatch; ++b) {
        if (rb + b < r1) {
          wd[b] = __ldcs(reinterpret_cast<const uint2*>(wp + (int64_t)(rb + b) * row_bytes));
          sc[b] = __ldg(sp + (int64_t)(rb + b) * nsb);
        } else {
          const uint32_t zero = (BITS == 4) ? 0x88888888u : 0x80808080u;  // code 0
          wd[b] = make_uint2(zero, zero);
          sc[b] = 0.0f;
        }
      }
    };
    auto compute = [&](int rb, const uint2 (&wd)[kClBatch], const float (&sc)[kClBatch]) {
#pragma unroll
      for (int b = 0; b < kClBatch; ++b) {
        uint64_t code[CPT / 2];
        decode_word2<BITS>(wd[b].x, code);
        decode_word2<BITS>(wd[b].y, code + 16 / BITS);
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
    for (int rb = r0; rb < r1; rb += 2 * kClBatch) {
      if (rb + kClBatch < r1) load(rb + kClBatch, wb, sb_);
      compute(rb, wa, sa_);
      if (rb + kClBatch >= r1) break;
      if (rb + 2 * kClBatch < r1) load(rb + 2 * kClBatch, wa, sa_);
      compute(rb + kClBatch, wb, sb_);
    }
  }
  // warp partials -> this CTA's partial
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
    float s = 0.0f;
#pragma unroll
    for (int w = 0; w < kClWarps; ++w) s = __fadd_rn(s, red[w * MT * kCols + i]);
    cta_part[i] = s;
  }
  // K-slices of the cluster -> y, each CTA finishing kCols / 8 columns
  cluster_sync_all();
  const uint32_t rank = cluster_rank();
  constexpr int kSlice = kCols / kClSplits;
  for (int i = threadIdx.x; i < MT * kSlice; i += blockDim.x) {
    const int m = i / kSlice, c = rank * kSlice + i % kSlice;
    const int col = c_cta + c;
    float s = 0.0f;
#pragma unroll
    for (uint32_t r = 0; r < kClSplits; ++r) s = __fadd_rn(s, ld_cluster_f32(cta_part + m * kCols + c, r));
    if (m < M && col < N) y[(int64_t)m * N + col] = s;
  }
  cluster_sync_all();  // keep this CTA's shared memory alive until all peers have read it
}

size_t cluster_smem(int bits, int mt, int krows) {
  const int cols = 32 * (kClLB * 8 / bits);
  return (size_t)(mt * krows + kClWarps * mt * cols + mt * cols) * sizeof(float);
}
