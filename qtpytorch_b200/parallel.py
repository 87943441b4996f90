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
the single-GPU ones.
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
    widths = {b - a for a, b in w.shards}
    if len(widths) != 1:
        raise NotImplementedError("uneven column shards need a variable-size gather")
    words, scales = gather_columns(c_packed, c_scales, M, w.world, group)
    return mx_tensor(words, scales, out_dt, torch.Size([M, w.N]), M * w.N, w.block)


def _all_gather(t: torch.Tensor, world: int, group) -> torch.Tensor:
    """[world, *t.shape]: one all-gather (into one buffer on NCCL)."""
    out = torch.empty((world,) + tuple(t.shape), dtype=t.dtype, device=t.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, t, group=group)
    else:
        dist.all_gather(list(out.unbind(0)), t, group=group)
    return out


def gather_columns(c_packed: torch.Tensor, c_scales: torch.Tensor, M: int, world: int,
                   group=None):
    """Assemble row-major packed C from equal column shards.

    Each rank holds C[:, n0:n1] packed row-major ([M, nl] codes as storage
    words, [M, nl/block] scales).  Because every shard width is a whole
    number of scale blocks, row m of C is the concatenation over ranks of
    their row m: gather [G, M, ...] and reorder to [M, G, ...].
    """
    gp = _all_gather(c_packed.contiguous(), world, group)
    gs = _all_gather(c_scales.contiguous(), world, group)
    words = gp.view(world, M, -1).transpose(0, 1).reshape(-1)
    scales = gs.view(world, M, -1).transpose(0, 1).reshape(-1)
    return words, scales


def sharded_quantize(x: torch.Tensor, dt, block: int, world: int, rank: int):
    """Row-sharded quantize: this rank's (packed, scales) for its block range of
    the flattened tensor, with no communication.  Concatenating the ranks'
    outputs in rank order gives exactly ``ops.quantize(x)``."""
    from .dtypes import get_mx_dtype
    dt = get_mx_dtype(dt)
    if dt.is_hadamard:
        raise NotImplementedError("row sharding of 'h' dtypes needs whole rows per rank")
    flat = x.reshape(-1)
    nb = -(-flat.numel() // block)
    b0, b1 = row_shard(nb, world, rank)
    part = flat[b0 * block: min(b1 * block, flat.numel())]
    packed, scales, _ = ops.quantize(part, dt, block)
    return packed, scales, (b0, b1)
