// Peer mappings for the column-sharded matmul's fused output gather: a rank
// opens its peers' output buffers (CUDA IPC handles exchanged on the host)
// with its own device current, so the mapping lives in this rank's context
// with peer access to the owner.  Plain device memory: no multicast object.
#include <string.h>

#include "mxb_common.cuh"

extern "C" {

int mxb_ipc_open(const void* handle, int64_t handle_bytes, void** base) {
  if (!handle || !base) return MXB_E_ARG;
  if (handle_bytes != (int64_t)sizeof(cudaIpcMemHandle_t)) return MXB_E_ARG;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof h);
  MXB_CUDA_TRY(cudaIpcOpenMemHandle(base, h, cudaIpcMemLazyEnablePeerAccess));
  return MXB_OK;
}

int mxb_ipc_close(void* base) {
  if (!base) return MXB_E_ARG;
  MXB_CUDA_TRY(cudaIpcCloseMemHandle(base));
  return MXB_OK;
}

}  // extern "C"
