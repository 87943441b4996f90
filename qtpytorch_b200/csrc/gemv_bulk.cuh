// Bulk-copy-staged split-K GEMV for int4 / int8 codes and M <= 2 (the
// decode case of configs[2]).  Included by gemv.cu inside its anonymous
// namespace.
//
// One producer warp streams 512-byte row slices of the packed W^T into a
// 4-stage shared-memory ring with cp.async.bulk (completion counted on an
// mbarrier per stage); 8 compute warps each take every 8th row of a stage,
// read 16 bytes per lane from shared memory, decode the codes exactly and
// accumulate with packed f32x2 FMA.  The load latency is covered by the
// ring, not by registers, so each SM keeps ~128 KB of weight in flight.
// Warp partials are added in a fixed order at the end; the K splits are
// added by split_reduce_kernel.  Every wait is bounded; on expiry the kernel
// records an error (read by mxb_device_error) and stops early.

__device__ int g_gemv_error = 0;

constexpr int kBulkWarps = 8;              // compute warps
constexpr int kBulkThreads = 32 * (kBulkWarps + 1);
constexpr int kBulkRowBytes = 512;         // one row slice of a CTA's columns
constexpr int kBulkStageRows = 32;
constexpr int kBulkStages = 4;
constexpr int kBulkStageBytes = kBulkStageRows * kBulkRowBytes;  // 16 KB
constexpr uint32_t kBulkSpin = 1u << 24;

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void bar_init(uint64_t* b, uint32_t n) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(b)), "r"(n));
}
__device__ __forceinline__ void bar_arrive(uint64_t* b) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(
                   smem_addr(b))
               : "memory");
}
__device__ __forceinline__ void bar_expect(uint64_t* b, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
          smem_addr(b)),
      "r"(bytes)
      : "memory");
}
__device__ __forceinline__ bool bar_wait(uint64_t* b, uint32_t parity) {
  for (uint32_t i = 0; i < kBulkSpin; ++i) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(b)), "r"(parity)
        : "memory");
    if (ok) return true;
  }
  atomicCAS(&g_gemv_error, 0, 1);
  return false;
}
// global -> shared bulk copy (16-byte aligned, size a multiple of 16), no multicast
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* b) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(b))
      : "memory");
}

template <int BITS, int MT, typename XT>
__global__ void __launch_bounds__(kBulkThreads) gemv_bulk_kernel(
    const XT* __restrict__ x, int M, int K, const uint8_t* __restrict__ W,
    const float* __restrict__ ws, int N, int block, int krows, float* __restrict__ part) {
  constexpr int CPT = 128 / BITS;      // columns per lane (16 bytes of codes)
  constexpr int kCols = 32 * CPT;      // columns of one CTA (512 bytes of codes)
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t* ring = smem;                                             // stages x 16 KB
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + kBulkStages * kBulkStageBytes);
  uint64_t* empty = full + kBulkStages;
  float* xs = reinterpret_cast<float*>(empty + kBulkStages);       // [MT][krows]
  float* red = reinterpret_cast<float*>(smem);  // reuses the ring after the K loop

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int k0 = blockIdx.y * krows;
  const int kn = min(krows, K - k0);
  const int c_cta = blockIdx.x * kCols;
  const int cols_here = min(kCols, N - c_cta);
  const int64_t row_bytes = (int64_t)N * BITS / 8;
  const int nstage = (kn + kBulkStageRows - 1) / kBulkStageRows;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kBulkStages; ++s) {
      bar_init(&full[s], 1);
      bar_init(&empty[s], kBulkWarps);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  for (int i = threadIdx.x; i < MT * krows; i += blockDim.x) {
    const int m = i / krows, kk = i % krows;
    xs[i] = (m < M && kk < kn) ? load_as_f32(x, (int64_t)m * K + k0 + kk) : 0.0f;
  }
  __syncthreads();

  uint64_t acc[MT][CPT / 2];
#pragma unroll
  for (int m = 0; m < MT; ++m)
#pragma unroll
    for (int c = 0; c < CPT / 2; ++c) acc[m][c] = 0ull;

  if (warp == kBulkWarps) {
    // producer: lane l copies row l of each stage
    const uint32_t slice = (uint32_t)cols_here * BITS / 8;
    const uint8_t* src0 = W + (int64_t)k0 * row_bytes + (int64_t)c_cta * BITS / 8;
    for (int st = 0; st < nstage; ++st) {
      const int s = st % kBulkStages, round = st / kBulkStages;
      if (round > 0 && !bar_wait(&empty[s], (round - 1) & 1)) break;
      const int rows = min(kBulkStageRows, kn - st * kBulkStageRows);
      if (lane == 0) bar_expect(&full[s], (uint32_t)rows * slice);
      __syncwarp();
      if (lane < rows)
        bulk_g2s(ring + s * kBulkStageBytes + lane * kBulkRowBytes,
                 src0 + (int64_t)(st * kBulkStageRows + lane) * row_bytes, slice, &full[s]);
    }
  } else {
    const int c0 = c_cta + lane * CPT;
    const bool active = c0 < N;
    const int64_t nsb = N / block;
    const float* sp = ws + (int64_t)k0 * nsb + (active ? c0 / block : 0);
    for (int st = 0; st < nstage; ++st) {
      const int s = st % kBulkStages, round = st / kBulkStages;
      const int rows = min(kBulkStageRows, kn - st * kBulkStageRows);
      float sc[kBulkStageRows / kBulkWarps];
#pragma unroll
      for (int j = 0; j < kBulkStageRows / kBulkWarps; ++j) {
        const int r = warp + j * kBulkWarps;
        sc[j] = (active && r < rows) ? __ldg(sp + (int64_t)(st * kBulkStageRows + r) * nsb) : 0.0f;
      }
      if (!bar_wait(&full[s], round & 1)) break;
      const uint8_t* stage = ring + s * kBulkStageBytes;
#pragma unroll
      for (int j = 0; j < kBulkStageRows / kBulkWarps; ++j) {
        const int r = warp + j * kBulkWarps;
        if (r < rows && active) {
          const uint4 v = *reinterpret_cast<const uint4*>(stage + r * kBulkRowBytes + lane * 16);
          const uint32_t wd[4] = {v.x, v.y, v.z, v.w};
          uint64_t code[CPT / 2];
#pragma unroll
          for (int q = 0; q < 4; ++q) decode_word2<BITS>(wd[q], code + q * (16 / BITS));
          const int kk = st * kBulkStageRows + r;
#pragma unroll
          for (int m = 0; m < MT; ++m) {
            const float xsv = __fmul_rn(xs[m * krows + kk], sc[j]);
            const uint64_t xs2 = pack2(xsv, xsv);
#pragma unroll
            for (int c = 0; c < CPT / 2; ++c) acc[m][c] = ffma2(xs2, code[c], acc[m][c]);
          }
        }
      }
      __syncwarp();
      if (lane == 0) bar_arrive(&empty[s]);
    }
  }
  __syncthreads();  // ring drained: reuse it for the warp partials
  if (warp < kBulkWarps) {
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
      for (int c = 0; c < CPT / 2; c += 2) {
        const float2 lo = unpack2(acc[m][c]), hi = unpack2(acc[m][c + 1]);
        *reinterpret_cast<float4*>(red + (warp * MT + m) * kCols + lane * CPT + 2 * c) =
            make_float4(lo.x, lo.y, hi.x, hi.y);
      }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < MT * kCols; i += blockDim.x) {
    const int m = i / kCols, c = i % kCols;
    const int col = c_cta + c;
    if (m >= M || col >= N) continue;
    float s = 0.0f;
#pragma unroll
    for (int w = 0; w < kBulkWarps; ++w) s = __fadd_rn(s, red[(w * MT + m) * kCols + c]);
    part[((int64_t)blockIdx.y * M + m) * N + col] = s;
  }
}

size_t bulk_smem(int mt, int krows) {
  const size_t ring = (size_t)kBulkStages * kBulkStageBytes;
  const size_t red = (size_t)kBulkWarps * mt * 32 * 32 * sizeof(float);  // CPT <= 32
  const size_t head = (ring > red ? ring : red) + 2 * kBulkStages * sizeof(uint64_t);
  return head + (size_t)mt * krows * sizeof(float);
}
