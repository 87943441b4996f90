// Peer mappings for the column-sharded matmul's fused output gather: a rank
// opens its peers' output buffers (CUDA IPC handles exchanged on the host)
// with its own device current, so the mapping lives in this rank's context
// with peer access to the owner.  Plain device memory: no multicast object.
#include <string.h>

#include "mxb_common.cuh"

namespace {

constexpr int kMaxRanks = 8;

// Where every rank's column shard of an int16d [M][N_full] output sits.
struct ColShards {
  const uint4* words[kMaxRanks];  // rank r's full-width codes (peer mapped)
  const float* scales[kMaxRanks];  // rank r's full-width scales [M][N_full / 128]
  int64_t off[kMaxRanks];          // first column of rank r's shard
  int64_t len[kMaxRanks];          // its width (columns, multiple of 128)
  int nranks, rank;
};

// Pull every peer's shard into this rank's output, the peers' memory read
// over NVLink by every SM: each thread moves 16-byte chunks (8 codes of one
// row), eight loads in flight before their stores.  Chunk index i of peer r
// is row i / (len / 8), chunk i % (len / 8).  Scales follow, one float per
// 128 columns of a row.
__global__ void __launch_bounds__(256) gather_cols_kernel(const __grid_constant__ ColShards g,
                                                          int64_t M, int64_t N_full,
                                                          uint4* __restrict__ out_words,
                                                          float* __restrict__ out_scales) {
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t nth = (int64_t)gridDim.x * blockDim.x;
  const int64_t row_chunks = N_full / 8;  // 16-byte chunks per output row
  for (int r = 0; r < g.nranks; ++r) {
    if (r == g.rank || g.len[r] == 0) continue;
    const int64_t per_row = g.len[r] / 8, c0 = g.off[r] / 8;
    const int64_t total = M * per_row;
    const uint4* src = g.words[r];
    for (int64_t i = tid; i < total; i += 8 * nth) {
      uint4 v[8];
      int64_t at[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int64_t j = i + u * nth;
        at[u] = -1;
        if (j < total) {
          at[u] = (j / per_row) * row_chunks + c0 + j % per_row;
          v[u] = __ldcs(src + at[u]);
        }
      }
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (at[u] >= 0) out_words[at[u]] = v[u];
    }
    const int64_t sb = g.len[r] / 128, s0 = g.off[r] / 128, nsb = N_full / 128;
    for (int64_t i = tid; i < M * sb; i += nth) {
      const int64_t at = (i / sb) * nsb + s0 + i % sb;
      out_scales[at] = __ldcs(g.scales[r] + at);
    }
  }
}

}  // namespace

extern "C" {

int mxb_allgather_cols(int nranks, int rank, int64_t M, int64_t N_full,
                       const int64_t* col_off, const int64_t* col_len,
                       void* const* out_words, float* const* out_scales, void* stream) {
  if (nranks < 1 || nranks > kMaxRanks || rank < 0 || rank >= nranks) return MXB_E_ARG;
  if (!col_off || !col_len || !out_words || !out_scales) return MXB_E_ARG;
  if (M <= 0 || N_full <= 0 || N_full % 128) return MXB_E_SHAPE;
  ColShards g;
  memset(&g, 0, sizeof g);
  g.nranks = nranks;
  g.rank = rank;
  for (int r = 0; r < nranks; ++r) {
    if (!out_words[r] || !out_scales[r] || ((uintptr_t)out_words[r] & 15)) return MXB_E_ARG;
    if (col_off[r] < 0 || col_len[r] < 0 || col_off[r] % 128 || col_len[r] % 128 ||
        col_off[r] + col_len[r] > N_full)
      return MXB_E_SHAPE;
    g.words[r] = static_cast<const uint4*>(out_words[r]);
    g.scales[r] = out_scales[r];
    g.off[r] = col_off[r];
    g.len[r] = col_len[r];
  }
  if (nranks == 1) return MXB_OK;
  gather_cols_kernel<<<4 * mxb::kSMs, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      g, M, N_full, static_cast<uint4*>(out_words[rank]), out_scales[rank]);
  MXB_LAUNCH_CHECK();
  return MXB_OK;
}

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
