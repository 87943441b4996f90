/*
 * mxb — B200 (sm_100a) kernels for the mxtorch quantize / pack / packed-matmul
 * hot path, behind a C ABI.
 *
 * Every entry point takes plain device pointers and sizes, runs on the CUDA
 * stream passed as `stream` (a cudaStream_t, or NULL for the legacy default
 * stream), returns an int status (MXB_OK or a negative MXB_E_* code, never
 * aborts) and allocates no device memory: the caller owns every buffer,
 * including the workspaces whose sizes the *_workspace_size functions report.
 * Calls are stateless and may run concurrently on different streams.
 *
 * Data layout (the reference's storage contract, mxtorch.py:870-985,
 * 1426-1528): a tensor of n elements is flattened row-major, zero-padded to
 * nb = ceil(n / block) blocks of `block` elements, and each block gets one
 * fp32 scale.  Codes are packed LSB-first as two's complement: 8/bits codes
 * per byte for bits in {1, 2, 4, 8}; 16-bit codes go two per int32 word, low
 * half first.  The packed buffer holds nb * block codes (padding included).
 * float4 ("float4d") codes are 4-bit indices into the sorted 16-entry grid
 * {±0, ±1/12, ±1/6, ±1/4, ±1/3, ±1/2, ±2/3, ±1}.
 */
#ifndef MXB_H_
#define MXB_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define MXB_OK 0
#define MXB_E_SHAPE (-1)     /* unsupported or inconsistent sizes */
#define MXB_E_DTYPE (-2)     /* unsupported bits / kind / variant combination */
#define MXB_E_ALIGN (-3)     /* a pointer is not aligned as the call requires */
#define MXB_E_CUDA (-4)      /* a CUDA runtime call or launch failed */
#define MXB_E_ARG (-6)       /* null pointer or invalid enum */
#define MXB_E_WORKSPACE (-7) /* workspace missing or too small */

/* input element types */
#define MXB_F32 0
#define MXB_BF16 1

/* code kinds */
#define MXB_KIND_INT 0   /* absmax integer codes (intNd) */
#define MXB_KIND_FLOAT 1 /* float4 grid-index codes (float4d) */

/* variants */
#define MXB_VAR_BASE 0
#define MXB_VAR_H 1 /* randomized Hadamard rotation of the last dim before quantizing */

/* weight-only matmul precision modes */
#define MXB_MODE_PARITY 0 /* fp32-faithful: |y - y_ref| <= 1e-5 * (|x| @ |W|) */
#define MXB_MODE_FAST 1   /* weights rounded to bf16 once: ~4e-3 relative per weight */

/* Library version (major * 10000 + minor * 100 + patch). */
int mxb_version(void);

/* Text of the last CUDA error seen by this thread ("" if none). */
const char* mxb_last_error(void);

/* Device-side error word of the current device: 0 if no kernel of this library
 * recorded a failure, else the code of the first bounded wait that gave up
 * (the kernel then returned early; its outputs are invalid).  Synchronises
 * the device.  clear != 0 resets the word. */
int mxb_device_error(int clear);

/* Number of kernels this library has launched in this process (all threads). */
uint64_t mxb_launch_count(void);

/* Bytes of packed storage for n codes of `bits` (1,2,4,8,16) at `block`. */
size_t mxb_packed_bytes(int64_t n, int bits, int block);

/* Workspace bytes mxb_quantize needs for these arguments (0 for the common
 * vectorised cases). */
size_t mxb_quantize_workspace_size(int64_t n, int64_t row_len, int bits, int kind,
                                   int variant, int block);

/*
 * Block-wise absmax quantize + bit-pack.
 * Replaces mxtorch `quantize` (mxtorch.py:1684-1763) for the base and "h"
 * variants, i.e. `_quant_int` (1426-1463), `_quant_float` (1465-1528),
 * `bit_packer.pack_auto` (976-980) and, for "h", `hadamard_rotation.rotate`
 * (2866-2890) along rows of `row_len` elements.
 *   x        device, n elements of x_dtype (MXB_F32 / MXB_BF16), row-major
 *   row_len  length of the last dim (the rotated dim for "h"; n for 1-D)
 *   bits     1, 2, 4 or 8 (kind INT) / 4 (kind FLOAT)
 *   signs    "h" only: pow2ceil(row_len) fp32 ±1 values
 *   packed   mxb_packed_bytes(n, bits, block) bytes
 *   scales   ceil(n / block) floats
 * Codes and scales are bit-identical to the reference's CPU path.
 */
int mxb_quantize(const void* x, int x_dtype, int64_t n, int64_t row_len, int bits,
                 int kind, int variant, int block, const float* signs, void* packed,
                 float* scales, void* workspace, size_t workspace_bytes, void* stream);

/* Workspace bytes mxb_dynamic_quantize needs (0 when block is 8..256). */
size_t mxb_dynamic_quantize_workspace_size(int64_t n, int64_t block);

/*
 * Dynamic (runtime) integer quantize over flat blocks of any length.
 * Replaces mxtorch `dynamic_quantize` (mxtorch.py:2665-2712): "per_token"
 * is block = the last dim (one scale per row), "per_tensor" block = n,
 * "per_block" block = the given block.  scale = max(amax, 1e-12) / max_int
 * (a true division), codes = round-half-even(x / scale), packed like
 * `bit_packer.pack_auto`.
 *   x        device, n elements of x_dtype (MXB_F32 / MXB_BF16)
 *   bits     2, 4, 8 or 16 (int1 has max_int 0 in the reference: rejected)
 *   packed   mxb_packed_bytes(n, bits, block) bytes
 *   scales   ceil(n / block) floats
 * Bit-identical to the reference's CPU arithmetic.
 */
int mxb_dynamic_quantize(const void* x, int x_dtype, int64_t n, int64_t block, int bits,
                         void* packed, float* scales, void* workspace, size_t workspace_bytes,
                         void* stream);

/*
 * Unpack + dequantize to fp32.
 * Replaces mxtorch `_dequant` (mxtorch.py:1530-1597).  bits may also be 16
 * (the int16d output of the int8 x int8 matmul).  For "h" the inverse
 * rotation (`hadamard_rotation.unrotate`, 2892-2904) runs along rows of
 * `row_len`, the dimension quantize rotated.
 *   out      n floats
 */
int mxb_dequantize(const void* packed, const float* scales, int64_t n, int64_t row_len,
                   int bits, int kind, int variant, int block, const float* signs,
                   float* out, void* stream);

/*
 * Dequantize + ReLU to fp32 (base variants): relu(_dequant(x)), NaN kept.
 * Replaces the epilogue of mxtorch `fused_linear_relu` (mxtorch.py:4012-4074,
 * `_k_dequant_relu` 3441-3456; the reference's CPU branch
 * F.relu(y.dequantize()) is the formula).  Arguments as mxb_dequantize.
 */
int mxb_dequantize_relu(const void* packed, const float* scales, int64_t n, int bits, int kind,
                        int block, float* out, void* stream);

/*
 * SiLU(dequant(gate)) * dequant(up) to fp32, SiLU(g) = g / (1 + exp(-g)).
 * Replaces mxtorch `fused_silu_and_mul` (mxtorch.py:4077-4109,
 * `_k_dequant_silu_and_mul` 3459-3479) for two packed operands of one dtype,
 * block and length n (base variants).
 */
int mxb_dequantize_silu_mul(const void* gate_packed, const float* gate_scales,
                            const void* up_packed, const float* up_scales, int64_t n, int bits,
                            int kind, int block, float* out, void* stream);

/* Randomized Hadamard transform of `rows` rows of length d (pow2ceil(d) <=
 * 32768), out-of-place or in place.  inverse=0: y = WHT(x * signs) / sqrt(n)
 * (hadamard_rotation.rotate, mxtorch.py:2866-2890); inverse=1:
 * y = WHT(x) / sqrt(n) * signs (unrotate, 2892-2904). */
int mxb_hadamard_rows(const float* x, int64_t rows, int64_t d, const float* signs,
                      int inverse, float* out, void* stream);

/* Cross-shard stage of a row WHT split over G column shards (G = 1, 2, 4
 * or 8), fused with the reorder of the gathered shards.  N = G * L columns,
 * column j = g * L + l; H_N = H_G (x) H_L.  `t` is the all-gather
 * [G][M][L] of each rank's t_g = WHT_L(y_g) / sqrt(L) (mxb_hadamard_rows
 * with unit signs); out[m][g*L + l] = (sum_h H_G[g, h] t_h[m][l]) / sqrt(G)
 * * signs[g*L + l], i.e. `hadamard_rotation.unrotate` of the full rows
 * (mxtorch.py:2892-2904) up to fp32 rounding order.  L % 4 == 0, pointers
 * 16-byte aligned.  No counterpart in the reference (it has no sharding). */
int mxb_hadamard_cross(const float* t, int64_t M, int64_t L, int G, const float* signs,
                       float* out, void* stream);

/* Workspace bytes for mxb_qgemm. */
size_t mxb_qgemm_workspace_size(int64_t M, int64_t K, int64_t N, int bits, int block);

/*
 * Packed integer matmul C = A @ B of two quantized matrices, requantized.
 * Replaces `_dispatch_qgemm` (mxtorch.py:5497-5573) -> `_qscale_matmul`
 * (1299-1385) + `bit_packer.pack_auto`.
 *   a_packed / a_scales  A [M, K], `bits` codes, a_nscales = ceil(M*K/block)
 *   b_packed / b_scales  B [K, N], b_nscales = ceil(K*N/block)
 * Per K-block kb: P = A[:, kb] @ B[kb, :] in exact integers, then
 * C = C + fl(fl(P * sa[m, kb]) * sb[kb, n]) in kb order, sa = a_scales viewed
 * [M, K/block] and sb = b_scales viewed [K/block, N] (the reference's layout;
 * all-ones when the scale count does not match that view).  C is then
 * requantized over flat blocks of `block` to `out_bits` codes
 * (cs = max(amax, 1e-12) / max_out, code = rint(clamp(C / cs))).
 *   out_bits  2, 4, 8 or 16 (the reference's choice: a.bits + b.bits), or 32
 *             for the fp32 C alone (no requantization; c_packed / c_scales unused)
 *   c_packed  mxb_packed_bytes(M*N, out_bits, block) bytes
 *   c_scales  ceil(M*N/block) floats
 *   c_f32     optional [M, N] fp32 C before requantization (may be NULL)
 */
int mxb_qgemm(const void* a_packed, const float* a_scales, int64_t a_nscales,
              const void* b_packed, const float* b_scales, int64_t b_nscales, int64_t M,
              int64_t K, int64_t N, int bits, int block, int out_bits, void* c_packed,
              float* c_scales, float* c_f32, void* workspace, size_t workspace_bytes,
              void* stream);

/* Workspace bytes for mxb_qgemm_kmajor. */
size_t mxb_qgemm_kmajor_workspace_size(int64_t M, int64_t K, int64_t N, int bits, int block);

/*
 * The packed integer matmul in "k-major" mode: B quantized along K.  The
 * reference's CPU matmul reads B's scales as b_scales viewed [K/block, N]
 * (mxtorch.py:1354-1355) although `quantize` lays them along B's flat rows,
 * so most elements of B meet another element's scale.  Here the caller
 * passes B^T [N, K] quantized flat (`mx_tensor.quantize(B.t())`): with
 * K % block == 0 every block is one column's K-block, its scale
 * bt_scales[n * K/block + kb] is that of every element it covers, and
 * C = sum_kb fl(fl(P * sa[m, kb]) * sb[n, kb]) is the quantized product
 * dequant(A) @ dequant(B) up to fp32 rounding (1-bit codes count as +-1,
 * their dequantized meaning; the reference's matmul sign-extends them to
 * 0 / -1).  No counterpart in the reference; same arguments,
 * requantization and result as mxb_qgemm otherwise.
 *   bt_packed / bt_scales  B^T [N, K], bt_nscales = N * K / block
 *   K % block == 0 and a_nscales == M * K / block, else MXB_E_SHAPE.
 */
int mxb_qgemm_kmajor(const void* a_packed, const float* a_scales, int64_t a_nscales,
                     const void* bt_packed, const float* bt_scales, int64_t bt_nscales,
                     int64_t M, int64_t K, int64_t N, int bits, int block, int out_bits,
                     void* c_packed, float* c_scales, float* c_f32, void* workspace,
                     size_t workspace_bytes, void* stream);

/*
 * One rank's share of a column-sharded packed matmul with the output
 * all-gather fused into the kernel.  The rank holds B's column shard
 * [K, N_local] (its slice of the B-scale view, as mxb_qgemm reads it) and
 * computes C[:, n_off : n_off + N_local] of the int16d result; the tcgen05
 * epilogue writes each tile's packed codes and scale straight into the
 * full-width outputs of all `nranks` ranks (this rank's own buffers and its
 * peers' over NVLink, e.g. CUDA IPC mappings), rows of N_full columns, so
 * no gather or reorder pass follows.  Output codes are int16d (the int8 x
 * int8 result dtype; narrower operands give int16d here as well).  The
 * caller makes the ranks' results visible to each other after the launch
 * (a barrier on the stream, e.g. a one-element NCCL all-reduce) and must
 * not let a rank write a buffer its peers are still reading (alternate two
 * output sets).  No counterpart in the reference.
 *   out_words[r]   rank r's M * N_full / 2 int32 words (16-byte aligned)
 *   out_scales[r]  rank r's M * N_full / 128 floats
 *   shapes: M, K, N_local multiples of 128, block 128, N_full % 128 == 0,
 *   n_off % 128 == 0, 1 <= nranks <= 8; otherwise MXB_E_SHAPE / MXB_E_ARG.
 *   Workspace: mxb_qgemm_workspace_size(M, K, N_local, bits, block).
 */
int mxb_qgemm_sharded(const void* a_packed, const float* a_scales, int64_t a_nscales,
                      const void* b_packed, const float* b_scales, int64_t b_nscales,
                      int64_t M, int64_t K, int64_t N_local, int bits, int block,
                      int64_t N_full, int64_t n_off, int nranks, void* const* out_words,
                      float* const* out_scales, void* workspace, size_t workspace_bytes,
                      void* stream);

/*
 * mxb_qgemm_sharded followed on the stream by the library's own cross-rank
 * completion barrier, so no collective is needed: when the call's work on
 * the stream is done, every rank's stores into this rank's output are
 * complete.  sync_blocks[r] is rank r's 16-word (128-byte, 8-byte aligned)
 * barrier block, this rank's own (sync_blocks[rank]) included, zeroed once
 * before the first call and left to the library afterwards; every rank
 * makes the same sequence of calls.  A one-thread kernel after the matmul
 * signals the call to every rank with a system-scope store and waits (at
 * most 2 s, then the device error word holds 6 and the output is invalid)
 * for all ranks' signals.  The counters live on the device, so a captured
 * CUDA graph replays correctly.  Other arguments and result as
 * mxb_qgemm_sharded.  No counterpart in the reference.
 */
int mxb_qgemm_sharded_sync(const void* a_packed, const float* a_scales, int64_t a_nscales,
                           const void* b_packed, const float* b_scales, int64_t b_nscales,
                           int64_t M, int64_t K, int64_t N_local, int bits, int block,
                           int64_t N_full, int64_t n_off, int nranks, int rank,
                           void* const* out_words, float* const* out_scales,
                           void* const* sync_blocks, void* workspace, size_t workspace_bytes,
                           void* stream);

/*
 * The cross-rank barrier of mxb_qgemm_sharded_sync on its own: when it has
 * run on every rank's stream, every rank's earlier work on its stream has
 * been reached (one-thread kernel, system-scope signals over the same
 * barrier blocks and call counters, bounded wait of 2 s, then the device
 * error word holds 6).  Every rank makes the same sequence of barrier and
 * sharded-matmul calls.  No counterpart in the reference (host plumbing for
 * the sharded matmul; it lines up the ranks before a timed step).
 */
int mxb_peer_barrier(int nranks, int rank, void* const* sync_blocks, void* stream);

/*
 * Output all-gather of a column-sharded matmul, pulled by this rank: every
 * peer's shard (columns col_off[r] .. col_off[r] + col_len[r] of every row)
 * is read from out_words[r] / out_scales[r] (peer memory over NVLink, e.g.
 * mxb_ipc_open mappings) into this rank's own out_words[rank] /
 * out_scales[rank] by every SM (16-byte loads, several in flight per thread); int16d
 * codes [M][N_full] as 32-bit words, scales [M][N_full / 128].  The peers'
 * shards must be complete before the launch (mxb_peer_barrier after their
 * mxb_qgemm_sharded with only their own output), and a rank must not
 * rewrite its shard while peers may still read it (alternate two output
 * sets).  Offsets and widths multiples of 128, 1 <= nranks <= 8.  No
 * counterpart in the reference (its matmul is single-device); the gather
 * step of the N-sharded matmul.
 */
int mxb_allgather_cols(int nranks, int rank, int64_t M, int64_t N_full,
                       const int64_t* col_off, const int64_t* col_len,
                       void* const* out_words, float* const* out_scales, void* stream);

/* Map a peer rank's device allocation into this process for the calling
 * thread's current device (cudaIpcOpenMemHandle with lazy peer access):
 * `handle` is the owner's cudaIpcMemHandle_t (handle_bytes == 64); *base
 * receives the mapped base address.  Host plumbing for mxb_qgemm_sharded's
 * output lists; no counterpart in the reference. */
int mxb_ipc_open(const void* handle, int64_t handle_bytes, void** base);
/* Unmap an address returned by mxb_ipc_open. */
int mxb_ipc_close(void* base);

/* Workspace bytes for mxb_linear_wonly. */
size_t mxb_linear_wonly_workspace_size(int64_t M, int64_t K, int64_t N, int bits,
                                       int kind, int block, int mode);

/*
 * Weight-only linear y = x @ dequant(W^T), fp32 output.
 * Replaces `mx_linear.forward` (mxtorch.py:7454-7473): the weight is stored
 * transposed, W^T [K = in, N = out], quantized flat (scale s[k, n // block]
 * when N % block == 0), and y = fp32(x) @ fl(code * s).
 *   x        [M, K] of x_dtype (MXB_F32 / MXB_BF16)
 *   w_packed / w_scales  the mx_tensor storage of W^T
 *   y        [M, N] fp32
 * Small M (decode) runs split-K: with bf16 x, integer codes and
 * block % 128 == 0, a tcgen05 kernel for 3 <= M <= 32 (the block scale
 * applied to x, the codes used as exact bf16 MMA operands); otherwise, for
 * M <= 16, a GEMV on the CUDA cores.  Larger M runs the tcgen05 GEMM.
 */
int mxb_linear_wonly(const void* x, int x_dtype, int64_t M, int64_t K, const void* w_packed,
                     const float* w_scales, int64_t N, int bits, int kind, int block,
                     int mode, float* y, void* workspace, size_t workspace_bytes,
                     void* stream);

/*
 * Weight-only linear with the weight stored K-major: y = x @ dequant(W)^T,
 * fp32 output.  Replaces the matmul of `mx_dynamic_linear.forward`
 * (mxtorch.py:8947-8978: tokens.float() @ w_mx.dequantize().t()), whose
 * weight is W [N = out, K = in] quantized flat along K (`mx_tensor.quantize(
 * linear.weight)`, 8929-8930), so element (n, k) has scale
 * w_scales[(n * K + k) / block].  No dequantized weight is materialised.
 *   x        [M, K] of x_dtype (MXB_F32 / MXB_BF16)
 *   w_packed / w_scales  the mx_tensor storage of W [N, K]
 *   y        [M, N] fp32
 * bf16 x with M > 16, K % 64 == 0, N % 128 == 0, K % block == 0 and 2-8 bit
 * codes runs the tcgen05 kernel (parity / fast modes as mxb_linear_wonly);
 * every other shape a CUDA-core kernel.  No workspace.
 */
int mxb_linear_wonly_kmajor(const void* x, int x_dtype, int64_t M, int64_t K,
                            const void* w_packed, const float* w_scales, int64_t N, int bits,
                            int kind, int block, int mode, float* y, void* stream);

/*
 * The decode (small-M) weight-only linear of mxb_linear_wonly, for callers
 * that cannot allocate device memory when they run the layer: runtimes that
 * only use buffers planned ahead of time, code inside a fixed memory pool,
 * or foreign-language hosts without a CUDA allocator.  It takes no
 * workspace; the split-K partial sums go to a 16 MiB array inside the
 * library (every GPU that loads the library keeps it until exit).
 * It has no counterpart in the reference; it exists only for such callers.
 *   Same arguments and result as mxb_linear_wonly for the split-K shapes
 *   (1 <= M <= 16, N % 8 == 0, N % block == 0, block % 8 == 0; with bf16 x,
 *   integer codes, block % 128 == 0, N % 128 == 0 and K % 64 == 0 also
 *   M up to 32); other shapes return MXB_E_SHAPE.  The split plan is the
 *   one mxb_linear_wonly uses, with its K splits made longer (up to the
 *   longest the planned kernel takes) until the partial sums, splits * M *
 *   N * 4 bytes, fit 16 MiB; shapes that still do not fit return
 *   MXB_E_WORKSPACE.
 *   The first call on each device looks the array up (with that device
 *   current); make that first call before any stream capture.  A device
 *   reset moves the array: the next call looks it up again.  All calls
 *   share the array: calls that may run at the same time on the GPU (other
 *   streams, other threads) race and must be serialized by the caller.
 *   Nothing in it needs clearing: each call writes every partial sum it reads.
 */
int mxb_linear_wonly_noalloc(const void* x, int x_dtype, int64_t M, int64_t K,
                             const void* w_packed, const float* w_scales, int64_t N, int bits,
                             int kind, int block, float* y, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MXB_H_ */
