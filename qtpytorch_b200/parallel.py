"""Multi-GPU layout of the hot path: one process per GPU, torch.distributed.

* quantize / dequantize are row-sharded: each rank owns whole scale blocks
  and no data crosses GPUs;
* the packed matmul and the weight-only linear are sharded along the output
  dimension N in whole 128-column blocks: each rank computes C[:, n0:n1]
  from the full A and its column shard of B, then one all-gather (NCCL over
  NVLink on B200 nodes, gloo on CPU test worlds) assembles C.

The packed matmul keeps the reference's B-scale view (b_scales viewed
[K/block, N], mxtorch.py:1354-1355): a rank's shard of that view is
``b_scales.view(K/block, N)[:, n0:n1]``, so sharded results are identical to
the single-GPU ones.  The weight-only linear stores W^T [K, N] quantized flat
with N % block == 0, so a shard of whole blocks is the column range of every
row's codes and of the scale matrix s[k, n / block]; ``h`` dtypes are
unrotated along the full rows of y after the gather.  Shards may differ by
one block (11008 = 86 blocks over 8 ranks): the gather pads every shard to
the widest one.
"""
from __future__ import annotations

from typing import List, Optional, Tuple

import torch
import torch.distributed as dist

from . import ops
from .dtypes import optimal_output_dtype
from .tensor import mx_tensor


def column_shards(N: int, world: int, unit: int = 128) -> List[Tuple[int, int]]:
    """Split N columns into ``world`` ranges of whole ``unit``-column blocks,
    as even as possible (earlier ranks take the remainder)."""
    if N % unit:
        raise ValueError(f"N={N} is not a multiple of {unit}")
    blocks = N // unit
    base, rem = divmod(blocks, world)
    out, b = [], 0
    for r in range(world):
        nb = base + (1 if r < rem else 0)
        out.append((b * unit, (b + nb) * unit))
        b += nb
    return out


def row_shard(n_blocks: int, world: int, rank: int) -> Tuple[int, int]:
    """Block range [b0, b1) of a row-sharded quantize."""
    base, rem = divmod(n_blocks, world)
    b0 = rank * base + min(rank, rem)
    return b0, b0 + base + (1 if rank < rem else 0)


class ShardedQGemmWeight:
    """The column shard of a quantized int matrix B [K, N] held by one rank."""

    def __init__(self, qb: mx_tensor, world: int, rank: int):
        K, N = qb._mx_orig_shape
        self.K, self.N, self.world, self.rank = K, N, world, rank
        self.block = qb._mx_block
        self.dtype = qb._mx_dtype
        if self.dtype.bits != 8:
            raise NotImplementedError("column sharding is implemented for int8 codes")
        self.shards = column_shards(N, world, self.block)
        n0, n1 = self.shards[rank]
        kbn = -(-K // self.block)
        self.n0, self.n1 = n0, n1
        self.codes = qb._mx_packed[: K * N].view(K, N)[:, n0:n1].contiguous()
        if qb._mx_scales.numel() == kbn * N:
            self.scales = qb._mx_scales.view(kbn, N)[:, n0:n1].contiguous()
        else:  # the reference then uses all-ones B scales
            self.scales = torch.ones(kbn, n1 - n0, device=qb._mx_packed.device)


def sharded_qgemm(qa: mx_tensor, w: ShardedQGemmWeight,
                  group: Optional[dist.ProcessGroup] = None) -> mx_tensor:
    """C = A @ B with B column-sharded over the ranks of ``group``."""
    M, K = qa._mx_orig_shape
    if K != w.K:
        raise ValueError("inner dimensions differ")
    out_dt = optimal_output_dtype("matmul", qa._mx_dtype, w.dtype)
    nl = w.n1 - w.n0
    c_packed, c_scales, _ = ops.qgemm(qa._mx_packed, qa._mx_scales, w.codes, w.scales, M, K,
                                      nl, 8, w.block, out_dt.bits)
    if w.world == 1:
        return mx_tensor(c_packed, c_scales, out_dt, torch.Size([M, w.N]), M * w.N, w.block)
    words, scales = gather_columns(c_packed, c_scales, M, w.world, group,
                                   widths=[b - a for a, b in w.shards], bits=out_dt.bits,
                                   block=w.block)
    return mx_tensor(words, scales, out_dt, torch.Size([M, w.N]), M * w.N, w.block)


class PeerOutputs:
    """Two sets of full-width int16d outputs (codes as int32 words, scales)
    of a column-sharded matmul, each visible to every rank.

    Every rank allocates its own buffers with torch; the CUDA IPC handles
    (torch's tensor sharing) are exchanged on the host and each rank maps its
    peers' buffers with its own device current (``mxb_ipc_open``): plain
    peer mappings, no multicast object.  Calls alternate between the two
    sets, so a rank that runs one call ahead never writes the set its peers
    may still be reading."""

    def __init__(self, M: int, N_full: int, block: int, world: int, rank: int, group=None,
                 device=None):
        from . import _lib as L
        import ctypes as C
        self.M, self.N, self.block, self.world, self.rank = M, N_full, block, world, rank
        dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        lib = L.load()
        self._opened = []
        self.sets = []
        # the in-kernel barrier's block of this rank (zeroed once), mapped by
        # every peer like the outputs
        self.sync = torch.zeros(16, dtype=torch.int64, device=dev)
        mine = self._share(self.sync)
        allh = [None] * world
        if world > 1:
            dist.all_gather_object(allh, mine, group=group)
        else:
            allh[0] = mine
        ptr_sync = []
        for r in range(world):
            if r == rank:
                ptr_sync.append(self.sync.data_ptr())
                continue
            handle, off = allh[r]
            base = C.c_void_p()
            with torch.cuda.device(dev):
                rc = lib.mxb_ipc_open(handle, len(handle), C.byref(base))
            L.check(rc, "mxb_ipc_open")
            self._opened.append(base.value)
            ptr_sync.append(base.value + off)
        self.ptr_sync = (C.c_void_p * world)(*ptr_sync)
        self._dev = dev
        for _ in range(2):
            words = torch.empty(M * N_full // 2, dtype=torch.int32, device=dev)
            scales = torch.empty(M * N_full // block, dtype=torch.float32, device=dev)
            mine = [self._share(t) for t in (words, scales)]
            allh = [None] * world
            if world > 1:
                dist.all_gather_object(allh, mine, group=group)
            else:
                allh[0] = mine
            ptr_w, ptr_s = [], []
            for r in range(world):
                if r == rank:
                    ptr_w.append(words.data_ptr())
                    ptr_s.append(scales.data_ptr())
                    continue
                got = []
                for handle, off in allh[r]:
                    base = C.c_void_p()
                    with torch.cuda.device(dev):
                        rc = lib.mxb_ipc_open(handle, len(handle), C.byref(base))
                    L.check(rc, "mxb_ipc_open")
                    self._opened.append(base.value)
                    got.append(base.value + off)
                ptr_w.append(got[0])
                ptr_s.append(got[1])
            self.sets.append({
                "words": words, "scales": scales,
                "ptr_w": (C.c_void_p * world)(*ptr_w), "ptr_s": (C.c_void_p * world)(*ptr_s)})
        self.i = 0

    def barrier(self) -> None:
        """Device-side barrier over the ranks' barrier blocks on the current
        stream (mxb_peer_barrier): every rank's earlier work on its stream
        has been reached when it completes.  Every rank calls it the same
        number of times, in the same order relative to the fused matmuls."""
        from . import _lib as L
        import ctypes as C
        lib = L.load()
        st = torch.cuda.current_stream(self._dev).cuda_stream
        L.check(lib.mxb_peer_barrier(self.world, self.rank, C.cast(self.ptr_sync, C.c_void_p),
                                     C.c_void_p(st)), "mxb_peer_barrier")

    @staticmethod
    def _share(t: torch.Tensor):
        """(cudaIpcMemHandle_t of t's CUDA allocation, byte offset of t in it).

        torch's storage sharing returns its own handle encoding: a version
        byte and a type byte ('c' for a cudaMalloc segment) before the
        64-byte CUDA IPC handle; other types (expandable segments) cannot be
        opened with cudaIpcOpenMemHandle and are refused."""
        st = t.untyped_storage()
        (_dev, handle, _size, storage_off, *_rest) = st._share_cuda_()
        h = bytes(handle)
        if len(h) == 66 and h[1] == ord("c"):
            h = h[2:]
        elif len(h) != 64:
            raise RuntimeError(f"unsupported CUDA IPC handle encoding ({len(h)} bytes, "
                               f"type {h[1:2]!r}); expandable segments cannot be mapped")
        return h, int(storage_off) + t.storage_offset() * t.element_size()

    def next(self):
        s = self.sets[self.i]
        self.i ^= 1
        return s

    def close(self):
        from . import _lib as L
        lib = L.load()
        for b in self._opened:
            lib.mxb_ipc_close(b)
        self._opened = []


def sharded_qgemm_pull(qa: mx_tensor, w: ShardedQGemmWeight, peers: PeerOutputs) -> mx_tensor:
    """C = A @ B with B column-sharded, gathered by pulling: each rank's
    GEMM writes its int16d tiles into its own full-width output only
    (mxb_qgemm_sharded with one output), the device barrier orders the
    ranks (mxb_peer_barrier), then every SM of each rank reads the peers'
    shards over NVLink into its own output (mxb_allgather_cols).  Same
    result as ``sharded_qgemm_fused``; no collective, graph-capturable."""
    from . import _lib as L
    import ctypes as C
    M, K = qa._mx_orig_shape
    if K != w.K:
        raise ValueError("inner dimensions differ")
    out_dt = optimal_output_dtype("matmul", qa._mx_dtype, w.dtype)
    if out_dt.bits != 16:
        raise NotImplementedError("the sharded gather writes int16d codes (int8 x int8)")
    nl = w.n1 - w.n0
    dev = qa._mx_packed.device
    lib = L.load()
    wsb = lib.mxb_qgemm_workspace_size(M, K, nl, w.dtype.bits, w.block)
    ws = L.workspace(wsb, dev)
    out = peers.next()
    own_w = (C.c_void_p * 1)(out["ptr_w"][w.rank])
    own_s = (C.c_void_p * 1)(out["ptr_s"][w.rank])
    offs = (C.c_int64 * w.world)(*[a for a, _ in w.shards])
    lens = (C.c_int64 * w.world)(*[b - a for a, b in w.shards])
    with torch.cuda.device(dev):
        rc = lib.mxb_qgemm_sharded(L.ptr(qa._mx_packed), L.ptr(qa._mx_scales),
                                   qa._mx_scales.numel(), L.ptr(w.codes), L.ptr(w.scales),
                                   w.scales.numel(), M, K, nl, w.dtype.bits, w.block, w.N,
                                   w.n0, 1, C.cast(own_w, C.c_void_p), C.cast(own_s, C.c_void_p),
                                   L.ptr(ws), wsb, L.stream_of(dev))
        L.check(rc, f"mxb_qgemm_sharded({M}x{K}x{nl} of {w.N}, own output)")
        if w.world > 1:
            peers.barrier()
            rc = lib.mxb_allgather_cols(w.world, w.rank, M, w.N, C.cast(offs, C.c_void_p),
                                        C.cast(lens, C.c_void_p),
                                        C.cast(out["ptr_w"], C.c_void_p),
                                        C.cast(out["ptr_s"], C.c_void_p), L.stream_of(dev))
            L.check(rc, "mxb_allgather_cols")
    return mx_tensor(out["words"], out["scales"], out_dt, torch.Size([M, w.N]), M * w.N, w.block)


def sharded_qgemm_fused(qa: mx_tensor, w: ShardedQGemmWeight, peers: PeerOutputs,
                        group=None, in_kernel_barrier: bool = True) -> mx_tensor:
    """C = A @ B with B column-sharded, the output all-gather fused into the
    GEMM kernel: every rank's epilogue writes its tiles' int16d codes and
    scales straight into all ranks' full-width outputs.  The ranks' writes
    are ordered before any rank reads either by the library's barrier kernel
    over peer-mapped flags (``in_kernel_barrier``, mxb_qgemm_sharded_sync:
    no collective, and the step can be captured in a CUDA graph) or by a
    one-element all-reduce on the stream after it (mxb_qgemm_sharded).  Same result as
    ``sharded_qgemm``; needs the tcgen05 shapes (M, K and every shard a
    multiple of 128, block 128)."""
    from . import _lib as L
    import ctypes as C
    M, K = qa._mx_orig_shape
    if K != w.K:
        raise ValueError("inner dimensions differ")
    out_dt = optimal_output_dtype("matmul", qa._mx_dtype, w.dtype)
    if out_dt.bits != 16:
        raise NotImplementedError("the fused gather writes int16d codes (int8 x int8)")
    nl = w.n1 - w.n0
    dev = qa._mx_packed.device
    lib = L.load()
    wsb = lib.mxb_qgemm_workspace_size(M, K, nl, w.dtype.bits, w.block)
    ws = L.workspace(wsb, dev)
    out = peers.next()
    with torch.cuda.device(dev):
        if in_kernel_barrier:
            rc = lib.mxb_qgemm_sharded_sync(
                L.ptr(qa._mx_packed), L.ptr(qa._mx_scales), qa._mx_scales.numel(),
                L.ptr(w.codes), L.ptr(w.scales), w.scales.numel(), M, K, nl, w.dtype.bits,
                w.block, w.N, w.n0, w.world, w.rank, C.cast(out["ptr_w"], C.c_void_p),
                C.cast(out["ptr_s"], C.c_void_p), C.cast(peers.ptr_sync, C.c_void_p),
                L.ptr(ws), wsb, L.stream_of(dev))
        else:
            rc = lib.mxb_qgemm_sharded(L.ptr(qa._mx_packed), L.ptr(qa._mx_scales),
                                       qa._mx_scales.numel(), L.ptr(w.codes), L.ptr(w.scales),
                                       w.scales.numel(), M, K, nl, w.dtype.bits, w.block, w.N,
                                       w.n0, w.world, C.cast(out["ptr_w"], C.c_void_p),
                                       C.cast(out["ptr_s"], C.c_void_p), L.ptr(ws), wsb,
                                       L.stream_of(dev))
    L.check(rc, f"mxb_qgemm_sharded({M}x{K}x{nl} of {w.N})")
    if w.world > 1 and not in_kernel_barrier:
        flag = torch.zeros(1, device=dev)
        dist.all_reduce(flag, group=group)  # every rank's kernel (and its peer stores) done
    return mx_tensor(out["words"], out["scales"], out_dt, torch.Size([M, w.N]), M * w.N, w.block)


class ShardedLinearWeight:
    """The column shard of an ``mx_linear`` weight (W^T [K, N] quantized flat,
    any code width) held by one rank: whole ``block``-column groups, so the
    shard is a column range of every row's codes and of s[k, n / block]."""

    def __init__(self, w: mx_tensor, world: int, rank: int):
        K, N = w._mx_orig_shape
        self.K, self.N, self.world, self.rank = K, N, world, rank
        self.block = w._mx_block
        self.dtype = w._mx_dtype
        if N % self.block or self.block % 8:
            raise ValueError("column sharding needs N % block == 0 and block % 8 == 0")
        self.shards = column_shards(N, world, max(self.block, 128))
        n0, n1 = self.shards[rank]
        self.n0, self.n1 = n0, n1
        bits = self.dtype.bits
        row = N * bits // 8
        self.codes = (w._mx_packed.view(torch.uint8)[: K * row].view(K, row)
                      [:, n0 * bits // 8: n1 * bits // 8].contiguous())
        nsb = N // self.block
        self.scales = (w._mx_scales[: K * nsb].view(K, nsb)
                       [:, n0 // self.block: n1 // self.block].contiguous())
        # ``h`` rows unrotate as local L-point transforms plus one G-point
        # stage across the shards when every shard has the same power-of-two
        # width L and N = G * L is a power of two (the Kronecker split)
        widths = {b - a for a, b in self.shards}
        L_ = n1 - n0
        self.kron_split = (self.dtype.is_hadamard and len(widths) == 1 and world in (1, 2, 4, 8)
                           and L_ & (L_ - 1) == 0 and L_ % 4 == 0)

    @classmethod
    def from_module(cls, m, world: int, rank: int) -> "ShardedLinearWeight":
        return cls(m._mx_weight, world, rank)


def sharded_linear(x: torch.Tensor, w: ShardedLinearWeight, group=None, mode: str = "parity",
                   out_dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """y = x @ dequant(W^T) with W^T column-sharded over the ranks of
    ``group`` (x replicated on every rank).  Each rank computes y[:, n0:n1]
    with the single-GPU kernel, then one all-gather assembles y; for ``h``
    dtypes the full rows are unrotated afterwards.  ``out_dtype`` bf16 casts
    before the gather (half the bytes on NVLink) unless the rows still need
    the fp32 unrotation."""
    from . import _lib as L
    lead = x.shape[:-1]
    K = x.shape[-1]
    if K != w.K:
        raise ValueError("inner dimensions differ")
    xm = x.reshape(-1, K)
    M = xm.shape[0]
    md = L.MODE_FAST if mode == "fast" else L.MODE_PARITY
    y = ops.linear_wonly(xm, w.codes, w.scales, K, w.n1 - w.n0, w.dtype, w.block, md)
    h = w.dtype.is_hadamard
    if h and w.kron_split and w.world > 1:
        # H_N = H_G (x) H_L: each rank transforms its own L columns, the one
        # all-gather moves those, and one kernel runs the G-point stage, the
        # signs and the reorder to row-major
        L_ = w.n1 - w.n0
        t = ops.hadamard_rows(y, None, inverse=True)
        if w.world > 1:
            t = _all_gather(t.contiguous(), w.world, group)  # [G, M, L]
        y = ops.hadamard_cross(t, M, L_, w.world, w.dtype.hadamard_seed)
        if out_dtype == torch.bfloat16:
            y = y.bfloat16()
        return y.reshape(*lead, w.N)
    if out_dtype == torch.bfloat16 and not h:
        y = y.bfloat16()
    if w.world > 1:
        y = gather_dense_columns(y, M, w.world, [b - a for a, b in w.shards], group)
    if h:
        y = ops.hadamard_rows(y, w.dtype.hadamard_seed, inverse=True)
        if out_dtype == torch.bfloat16:
            y = y.bfloat16()
    return y.reshape(*lead, w.N)


def _all_gather(t: torch.Tensor, world: int, group) -> torch.Tensor:
    """[world, *t.shape]: one all-gather (into one buffer on NCCL)."""
    out = torch.empty((world,) + tuple(t.shape), dtype=t.dtype, device=t.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, t, group=group)
    else:
        dist.all_gather(list(out.unbind(0)), t, group=group)
    return out


def _gather_rows_var(t: torch.Tensor, M: int, world: int, widths: List[int], group):
    """t [M, widths[rank]] on each rank -> [M, sum(widths)] (columns in rank
    order): every shard is padded to the widest, gathered once, then each
    rank's valid columns are concatenated per row."""
    wmax = max(widths)
    t = t.reshape(M, -1)
    if t.shape[1] < wmax:
        t = torch.cat([t, t.new_zeros(M, wmax - t.shape[1])], dim=1)
    g = _all_gather(t.contiguous(), world, group)  # [G, M, wmax]
    if all(w == wmax for w in widths):
        return g.transpose(0, 1).reshape(M, -1)
    return torch.cat([g[r, :, : widths[r]] for r in range(world)], dim=1)


def gather_dense_columns(y: torch.Tensor, M: int, world: int, widths: List[int],
                         group=None) -> torch.Tensor:
    """Assemble y [M, N] from the ranks' column shards y[:, n0:n1]."""
    return _gather_rows_var(y, M, world, widths, group)


def gather_columns(c_packed: torch.Tensor, c_scales: torch.Tensor, M: int, world: int,
                   group=None, widths: Optional[List[int]] = None, bits: int = 16,
                   block: int = 128):
    """Assemble row-major packed C from column shards.

    Each rank holds C[:, n0:n1] packed row-major ([M, nl] codes as storage
    words, [M, nl/block] scales).  Because every shard width is a whole
    number of scale blocks, row m of C is the concatenation over ranks of
    their row m: gather [G, M, ...] and reorder to [M, G, ...].  ``widths``
    (columns per rank) may differ by whole blocks; shards are then padded to
    the widest for the gather.
    """
    if widths is None or len(set(widths)) == 1:
        gp = _all_gather(c_packed.contiguous(), world, group)
        gs = _all_gather(c_scales.contiguous(), world, group)
        words = gp.view(world, M, -1).transpose(0, 1).reshape(-1)
        scales = gs.view(world, M, -1).transpose(0, 1).reshape(-1)
        return words, scales
    per_word = 2 if bits == 16 else 8 // bits  # codes per storage element
    words = _gather_rows_var(c_packed, M, world, [w // per_word for w in widths], group)
    scales = _gather_rows_var(c_scales, M, world, [w // block for w in widths], group)
    return words.reshape(-1), scales.reshape(-1)


def sharded_quantize(x: torch.Tensor, dt, block: int, world: int, rank: int):
    """Row-sharded quantize: this rank's (packed, scales) for its block range of
    the flattened tensor, with no communication.  Concatenating the ranks'
    outputs in rank order gives exactly ``ops.quantize(x)``.

    ``h`` dtypes rotate whole rows of the last dim (mxtorch.py:1720-1736), so
    their shards are whole rows, in units of the fewest rows that also end on
    a block boundary (lcm(row, block) elements); the returned range is then
    in blocks as well."""
    from .dtypes import get_mx_dtype
    dt = get_mx_dtype(dt)
    if dt.is_hadamard:
        return _sharded_quantize_rows(x, dt, block, world, rank)
    flat = x.reshape(-1)
    nb = -(-flat.numel() // block)
    b0, b1 = row_shard(nb, world, rank)
    part = flat[b0 * block: min(b1 * block, flat.numel())]
    packed, scales, _ = ops.quantize(part, dt, block)
    return packed, scales, (b0, b1)


def h_row_range(shape, block: int, bits: int, world: int, rank: int) -> Tuple[int, int]:
    """Rows [r0, r1) of an ``h`` tensor's last-dim rows held by ``rank``: whole
    rows, in units of lcm(row, block) elements so every shard starts on a
    block (and byte) boundary."""
    import math
    d = ops.row_len_of(shape)
    n = 1
    for s in shape:
        n *= int(s)
    rows = n // d if d else 0
    unit = math.lcm(d, block) // d  # rows per unit: whole rows ending on a block boundary
    if (unit * d * bits) % 8:
        raise ValueError("row shards of this width do not end on a whole byte")
    u0, u1 = row_shard(-(-rows // unit), world, rank)
    return min(u0 * unit, rows), min(u1 * unit, rows)


def _sharded_quantize_rows(x: torch.Tensor, dt, block: int, world: int, rank: int):
    d = ops.row_len_of(x.shape)
    rows = x.numel() // d if d else 0
    r0, r1 = h_row_range(x.shape, block, dt.bits, world, rank)
    part = x.reshape(rows, d)[r0:r1]
    packed, scales, _ = ops.quantize(part, dt, block)
    b0 = r0 * d // block
    return packed, scales, (b0, b0 + scales.numel())
