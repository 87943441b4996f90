// Walsh-Hadamard transform of one row of n = 256 * V floats held in the
// registers of a 256-thread CTA (V values per thread), for the row lengths
// of the Hadamard variants' hot cases (n = 2048 .. 16384; configs[3] rotates
// rows of 8192).
//
// The stage order is the reference's (mxtorch.py:2811-2832): the stride-n/2
// stage first, down to stride 1, each pair (e, o) -> (e + o, e - o), so the
// results are bit-identical to the shared-memory transform.  Index bits are
// split hi | mid | lo, hi and mid log2(V) bits each and lo the low
// LB = 8 - log2(V):
//   phase A  thread t owns indices t + 256 j: the hi stages on j, in
//            registers;
//   phase B  through shared memory, thread t = (hi, lo) owns mid = 0..V-1:
//            the mid stages in registers;
//   phase C  (V >= 16) through shared memory again, thread t owns V / 2^LB
//            runs of 2^LB consecutive indices: the lo stages in registers,
//            and the row leaves in runs (vector stores, block-wise
//            quantization straight from registers).  For V = 8 the lo stages
//            run across the lanes of a warp instead (shuffles).
// Shared memory carries 2^LB floats of padding per 256, which keeps every
// pass free of bank conflicts.
#pragma once

namespace mxb {
namespace whtr {

template <int V>
struct Row {
  static constexpr int kLV = V == 8 ? 3 : V == 16 ? 4 : V == 32 ? 5 : 6;
  static constexpr int kN = 256 * V;
  static constexpr int kLB = 8 - kLV;     // low index bits
  static constexpr int kG = 1 << kLB;     // run length of phase C; padding per 256
  static constexpr int kRuns = V / kG;    // runs per thread in phase C (V >= 16)
  static constexpr bool kPhaseC = V >= 16;
  static constexpr int kSmemFloats = kN + (kN / 256) * kG;
  static_assert(V == 8 || V == 16 || V == 32 || V == 64, "V");

  __device__ static int pad(int i) { return i + (i >> 8) * kG; }
  // phase-A index of slot j of thread t
  __device__ static int idxA(int t, int j) { return t + 256 * j; }
  // phase-B index of slot m of thread t
  __device__ static int idxB(int t, int m) {
    const int lo = t & (kG - 1), hi = t >> kLB;
    return (hi << 8) | (m << kLB) | lo;
  }
  // final index of slot j: phase C (run j / kG, element j % kG) or phase B
  __device__ static int idx(int t, int j) {
    if constexpr (kPhaseC) return ((t + 256 * (j / kG)) << kLB) | (j % kG);
    return idxB(t, j);
  }

  template <int NV>
  __device__ static void stages_regs(float* v) {
#pragma unroll
    for (int h = NV / 2; h >= 1; h /= 2) {
#pragma unroll
      for (int j = 0; j < NV; ++j) {
        if (!(j & h)) {
          const float e = v[j], o = v[j + h];
          v[j] = __fadd_rn(e, o);
          v[j + h] = __fsub_rn(e, o);
        }
      }
    }
  }

  // Runs (the final layout) -> phase-A slots, through shared memory, for
  // rows that are loaded in runs of consecutive elements (vector loads).
  // Begins and ends with __syncthreads.
  __device__ static void from_runs(float (&v)[V], float* s) {
    static_assert(kPhaseC, "runs exist for V >= 16");
    const int t = threadIdx.x;
    __syncthreads();
#pragma unroll
    for (int r = 0; r < kRuns; ++r) {
      float4* p = reinterpret_cast<float4*>(s + pad((t + 256 * r) << kLB));
#pragma unroll
      for (int q = 0; q < kG / 4; ++q)
        p[q] = make_float4(v[r * kG + 4 * q], v[r * kG + 4 * q + 1], v[r * kG + 4 * q + 2],
                           v[r * kG + 4 * q + 3]);
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < V; ++j) v[j] = s[pad(idxA(t, j))];
    __syncthreads();
  }

  // v: phase-A slots on entry, final slots (idx) on exit.  `s` holds
  // kSmemFloats; the function begins and ends with __syncthreads.
  __device__ static void transform(float (&v)[V], float* s) {
    const int t = threadIdx.x;
    stages_regs<V>(v);  // index bits L-1 .. 8
    __syncthreads();
#pragma unroll
    for (int j = 0; j < V; ++j) s[pad(idxA(t, j))] = v[j];
    __syncthreads();
#pragma unroll
    for (int m = 0; m < V; ++m) v[m] = s[pad(idxB(t, m))];
    stages_regs<V>(v);  // index bits 7 .. kLB
    if constexpr (kPhaseC) {
      __syncthreads();
#pragma unroll
      for (int m = 0; m < V; ++m) s[pad(idxB(t, m))] = v[m];
      __syncthreads();
#pragma unroll
      for (int r = 0; r < kRuns; ++r) {
        const float4* p = reinterpret_cast<const float4*>(s + pad((t + 256 * r) << kLB));
#pragma unroll
        for (int q = 0; q < kG / 4; ++q) {
          const float4 a = p[q];
          v[r * kG + 4 * q] = a.x;
          v[r * kG + 4 * q + 1] = a.y;
          v[r * kG + 4 * q + 2] = a.z;
          v[r * kG + 4 * q + 3] = a.w;
        }
        stages_regs<kG>(v + r * kG);  // index bits kLB-1 .. 0
      }
    } else {
      const int lane = t & 31;
#pragma unroll
      for (int h = kG / 2; h >= 1; h /= 2) {  // index bits kLB-1 .. 0
#pragma unroll
        for (int m = 0; m < V; ++m) {
          const float p = __shfl_xor_sync(0xffffffffu, v[m], h);
          v[m] = (lane & h) ? __fsub_rn(p, v[m]) : __fadd_rn(v[m], p);
        }
      }
    }
    __syncthreads();
  }
};

// x / c rounded to nearest even, c = fl32(sqrt(n)):
//   mode 1  c a power of two: x * (1/c) is exact;
//   mode 2  q0 = x * r, e = fma(-q0, c, x), q = fma(e, r, q0) with
//           r = RN(1/c): Markstein's correction of the reciprocal product
//           (P. Markstein, IA-64 and Elementary Functions, 2000).  Checked
//           equal to the IEEE quotient on a B200 for every finite float
//           |x| >= 1e-30 at c = fl32(sqrt(2^l)), l = 3, 5, .., 15 (the host
//           selects it only there); smaller |x| (where the residual can
//           underflow), inf and NaN take the IEEE division;
//   mode 0  the IEEE division.
__device__ __forceinline__ float div_sqrtn(float x, float c, float r, int mode) {
  if (mode == 1) return __fmul_rn(x, r);
  const float ax = fabsf(x);
  if (mode == 2 && ax >= 1e-30f && ax <= 3.4028235e38f) {
    const float q0 = __fmul_rn(x, r);
    const float e = __fmaf_rn(-q0, c, x);
    return __fmaf_rn(e, r, q0);
  }
  return __fdiv_rn(x, c);
}

}  // namespace whtr
}  // namespace mxb
