// tcgen05 GEMM kernels (placeholder: routing disabled until the kernels land).
#include "mxb_common.cuh"
#include "mxb_internal.h"

namespace mxb {

bool tc_qgemm_eligible(int64_t, int64_t, int64_t, int, int, bool, bool, const void*,
                       const void*, const float*) {
  return false;
}
size_t tc_qgemm_workspace(int64_t, int64_t, int64_t, int) { return 0; }
int tc_qgemm(const void*, const float*, const void*, const float*, int64_t, int64_t, int64_t,
             int, int, float*, void*, size_t, cudaStream_t) {
  return MXB_E_SHAPE;
}

}  // namespace mxb
