// Decode-regime weight-only linear without any caller-supplied workspace.
//
// mxb_linear_wonly needs a workspace for the split-K partial sums, which the
// caller allocates.  Some callers cannot allocate device memory at the point
// where they run the layer: a host runtime that only hands out buffers it
// planned ahead of time, code running inside a pre-sized memory pool, or an
// FFI caller (Go, Java, ...) that has no CUDA allocator of its own.  This
// variant keeps the partial sums in a fixed array that lives in the library
// itself, so the caller passes only x, the packed weight and y.
#include "mxb_common.cuh"
#include "mxb_internal.h"

#include <mutex>

namespace {

// Partial-sum scratch shared by every call on a device: 16 MiB.  Each GPU
// that loads the library holds it until the process exits.
constexpr size_t kScratchBytes = 16u << 20;
static __device__ __align__(256) float g_gemv_scratch[kScratchBytes / sizeof(float)];

constexpr int kMaxDevices = 64;

// cuCtxGetCurrent / cuCtxGetId through the runtime's driver entry point (no
// libcuda link): the id of the device's current context, which changes when
// the context is destroyed and made again (cudaDeviceReset), the one event
// that moves the module's device array.
typedef int (*CtxGetCurrentFn)(void**);
typedef int (*CtxGetIdFn)(void*, unsigned long long*);

bool current_ctx_id(unsigned long long* id) {  // called under scratch_ptr's lock
  static CtxGetCurrentFn get_cur = nullptr;
  static CtxGetIdFn get_id = nullptr;
  static bool looked = false;
  if (!looked) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_cur = reinterpret_cast<CtxGetCurrentFn>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<CtxGetIdFn>(p);
    looked = true;
  }
  void* ctx = nullptr;
  if (!get_cur || !get_id || get_cur(&ctx) != 0 || ctx == nullptr) return false;
  return get_id(ctx, id) == 0;
}

// Device address of g_gemv_scratch, looked up with the device current and
// cached per device together with the id of the context it was looked up
// in; a new context (after a device reset) looks it up again.  In host code
// the symbol itself is only a host-side stand-in and must never be passed
// to a kernel.
float* scratch_ptr(int dev, int* rc) {
  static std::mutex mu;
  static float* ptrs[kMaxDevices] = {};
  static unsigned long long ctx_ids[kMaxDevices] = {};
  if (dev < 0 || dev >= kMaxDevices) {
    *rc = MXB_E_ARG;
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  unsigned long long id = 0;
  const bool have_id = current_ctx_id(&id);
  if (ptrs[dev] == nullptr || !have_id || ctx_ids[dev] != id) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_gemv_scratch);
    if (e != cudaSuccess) {
      mxb_set_cuda_error(e);
      *rc = MXB_E_CUDA;
      return nullptr;
    }
    ptrs[dev] = static_cast<float*>(p);
    ctx_ids[dev] = have_id ? id : 0;
  }
  *rc = MXB_OK;
  return ptrs[dev];
}

}  // namespace

extern "C" int mxb_linear_wonly_noalloc(const void* x, int x_dtype, int64_t M, int64_t K,
                                        const void* w_packed, const float* w_scales, int64_t N,
                                        int bits, int kind, int block, float* y,
                                        void* stream) {
  if (kind == MXB_KIND_FLOAT ? bits != 4
                             : !(bits == 1 || bits == 2 || bits == 4 || bits == 8))
    return MXB_E_DTYPE;
  if (kind != MXB_KIND_INT && kind != MXB_KIND_FLOAT) return MXB_E_DTYPE;
  if (x_dtype != MXB_F32 && x_dtype != MXB_BF16) return MXB_E_DTYPE;
  if (M < 0 || K <= 0 || N <= 0 || block <= 0) return MXB_E_SHAPE;
  if (M == 0) return MXB_OK;
  if (K * N >= (int64_t)1 << 31) return MXB_E_SHAPE;
  if (!x || !w_packed || !w_scales || !y) return MXB_E_ARG;

  mxb::GemvPlan plan = mxb::gemv_plan(M, K, N, bits, kind, block, w_packed, y, x_dtype, x);
  if (!plan.ok) return MXB_E_SHAPE;  // not a split-K (decode) shape
  // Fewer, longer K splits (up to the longest the planned kernel takes)
  // until the partial sums fit the fixed scratch.
  const int max_rows = plan.max_krows;
  while (plan.ws_bytes > kScratchBytes && plan.krows < max_rows) {
    int64_t krows = plan.krows * 2 > max_rows ? max_rows : plan.krows * 2;
    plan.krows = (int)krows;
    plan.splits = (int)mxb::cdiv(K, krows);
    plan.ws_bytes = (size_t)plan.splits * M * N * sizeof(float);
  }
  if (plan.ws_bytes > kScratchBytes) return MXB_E_WORKSPACE;  // beyond the 16 MiB maximum

  int dev = 0;
  MXB_CUDA_TRY(cudaGetDevice(&dev));
  int rc = MXB_OK;
  float* scratch = scratch_ptr(dev, &rc);
  if (rc != MXB_OK) return rc;
  // Every partial sum is written before it is read, so nothing is cleared.
  return mxb::gemv_run(plan, x, x_dtype, M, K, w_packed, w_scales, N, bits, kind, block, y,
                       scratch, static_cast<cudaStream_t>(stream));
}
