"""Multi-process host logic of the N-sharded matmul and the row-sharded
quantize, on CPU with world_size-2 gloo ranks.

The GPU kernel of each rank is stood in for by the CPU oracle (the checker),
so these tests cover the sharding, the reference's B-scale view per shard,
the all-gather and the reorder: the assembled packed result must be
identical to the unsharded one.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import mx_oracle as O
from qtpytorch_b200 import parallel as P
from qtpytorch_b200.dtypes import int8d
from qtpytorch_b200.tensor import mx_tensor

WORLD = 2


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _inputs(M=64, K=256, N=512):
    g = torch.Generator().manual_seed(7)
    return torch.randn(M, K, generator=g), torch.randn(K, N, generator=g)


def _qgemm_rank(rank, port, result_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        a, b = _inputs()
        M, K = a.shape
        N = b.shape[1]
        pa, sa, _ = O.quantize(a.numpy(), 8, "int", 128)
        pb, sb, _ = O.quantize(b.numpy(), 8, "int", 128)
        qb = mx_tensor(torch.from_numpy(pb), torch.from_numpy(sb), int8d, (K, N), K * N, 128)
        w = P.ShardedQGemmWeight(qb, WORLD, rank)
        nl = w.n1 - w.n0
        # this rank's shard computed by the oracle in place of the GPU kernel
        codes, cs, _ = O.qscale_matmul(O.unpack(pa, 8, M * K), sa, w.codes.numpy().reshape(-1),
                                       w.scales.numpy().reshape(-1), M, K, nl, 128, 16)
        words, scales = P.gather_columns(torch.from_numpy(O.pack(codes, 16)),
                                         torch.from_numpy(cs), M, WORLD)
        if rank == 0:
            result_q.put((words.numpy(), scales.numpy()))
    finally:
        dist.destroy_process_group()


def test_sharded_qgemm_gathers_identical_result():
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_qgemm_rank, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    words, scales = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    a, b = _inputs()
    M, K = a.shape
    N = b.shape[1]
    pa, sa, _ = O.quantize(a.numpy(), 8, "int", 128)
    pb, sb, _ = O.quantize(b.numpy(), 8, "int", 128)
    codes, cs, _ = O.qscale_matmul(O.unpack(pa, 8, M * K), sa, O.unpack(pb, 8, K * N), sb,
                                   M, K, N, 128, 16)
    assert np.array_equal(words, O.pack(codes, 16))
    assert np.array_equal(scales.view(np.uint32), cs.view(np.uint32))


def test_column_and_row_shards():
    assert P.column_shards(4096, 8) == [(i * 512, (i + 1) * 512) for i in range(8)]
    sh = P.column_shards(11008, 8)  # 86 blocks: 11,11,11,11,11,11,10,10
    assert [(b - a) // 128 for a, b in sh] == [11] * 6 + [10] * 2
    assert sh[0][0] == 0 and sh[-1][1] == 11008
    with pytest.raises(ValueError):
        P.column_shards(1000, 2)
    parts = [P.row_shard(10, 3, r) for r in range(3)]
    assert parts == [(0, 4), (4, 7), (7, 10)]


def test_row_sharded_quantize_concatenates_to_full():
    # the block ranges of the ranks tile the tensor; concatenating the ranks'
    # packed bytes and scales (oracle stand-in) reproduces the full quantize
    x = np.random.default_rng(3).standard_normal(10 * 128 + 37).astype(np.float32)
    full_p, full_s, _ = O.quantize(x, 4, "int", 128)
    nb = -(-x.size // 128)
    ps, ss = [], []
    for r in range(3):
        b0, b1 = P.row_shard(nb, 3, r)
        p, s, _ = O.quantize(x[b0 * 128: min(b1 * 128, x.size)], 4, "int", 128)
        ps.append(p)
        ss.append(s)
    assert np.array_equal(np.concatenate(ps), full_p)
    assert np.array_equal(np.concatenate(ss), full_s)


# ── weight-only linear, column-sharded (configs[3] layout), uneven shards ──

def _linear_inputs(dt_name, M=6, K=256, N=640):
    g = torch.Generator().manual_seed(11)
    w = torch.randn(N, K, generator=g) * 0.02
    x = torch.randn(M, K, generator=g)
    return x, w


def _w_mx(dt_name, w, block=128):
    """mx_linear's stored weight (W^T quantized flat) built with the oracle."""
    from qtpytorch_b200.dtypes import get_mx_dtype
    from qtpytorch_b200.hadamard import sign_vector
    dt = get_mx_dtype(dt_name)
    wt = w.t().contiguous().numpy()
    signs = sign_vector(wt.shape[-1], dt.hadamard_seed).numpy() if dt.is_hadamard else None
    p, s, n = O.quantize(wt, dt.bits, dt.kind, block, dt.is_hadamard, signs)
    return mx_tensor(torch.from_numpy(p), torch.from_numpy(s), dt, wt.shape, n, block), signs


def _shard_y(x, codes, scales, dt, K, nl, block):
    """A rank's y[:, n0:n1] (oracle stand-in for the GPU kernel): float64
    product of x and the shard's dequantized columns, rounded to fp32."""
    wdq = O.dequant_flat(codes.numpy().reshape(-1), scales.numpy().reshape(-1), dt.bits,
                         dt.kind, K * nl, block).reshape(K, nl)
    return torch.from_numpy((x.numpy().astype(np.float64) @ wdq.astype(np.float64))
                            .astype(np.float32))


def _linear_rank(rank, port, dt_name, result_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        x, w = _linear_inputs(dt_name)
        qw, signs = _w_mx(dt_name, w)
        sw = P.ShardedLinearWeight(qw, WORLD, rank)
        K, N = sw.K, sw.N
        nl = sw.n1 - sw.n0
        y_local = _shard_y(x, sw.codes, sw.scales, sw.dtype, K, nl, sw.block)
        y = P.gather_dense_columns(y_local, x.shape[0], WORLD,
                                   [b - a for a, b in sw.shards])
        if sw.dtype.is_hadamard:
            y = torch.from_numpy(O.unrotate(y.numpy(), signs))
        if rank == 0:
            result_q.put((y.numpy(), sw.shards))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("dt_name", ["int4d", "int2d", "int4dh"])
def test_sharded_linear_uneven_shards_match_full(dt_name):
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_linear_rank, args=(r, port, dt_name, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    y, shards = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert [(b - a) // 128 for a, b in shards] == [3, 2]  # 5 blocks over 2 ranks
    # the full weight's columns, computed shard range by shard range
    x, w = _linear_inputs(dt_name)
    qw, signs = _w_mx(dt_name, w)
    K, N = qw._mx_orig_shape
    full = O.dequant_flat(qw._mx_packed.numpy(), qw._mx_scales.numpy(), qw._mx_dtype.bits,
                          qw._mx_dtype.kind, K * N, 128).reshape(K, N)
    parts = [(x.numpy().astype(np.float64) @ full[:, a:b].astype(np.float64)).astype(np.float32)
             for a, b in shards]
    ref = np.concatenate(parts, axis=1)
    if qw._mx_dtype.is_hadamard:
        ref = O.unrotate(ref, signs)
    assert np.array_equal(y.view(np.uint32), ref.view(np.uint32))


def _qgemm_uneven_rank(rank, port, result_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        a, b = _inputs(M=32, K=256, N=640)
        M, K = a.shape
        N = b.shape[1]
        pa, sa, _ = O.quantize(a.numpy(), 8, "int", 128)
        pb, sb, _ = O.quantize(b.numpy(), 8, "int", 128)
        qb = mx_tensor(torch.from_numpy(pb), torch.from_numpy(sb), int8d, (K, N), K * N, 128)
        w = P.ShardedQGemmWeight(qb, WORLD, rank)
        nl = w.n1 - w.n0
        codes, cs, _ = O.qscale_matmul(O.unpack(pa, 8, M * K), sa, w.codes.numpy().reshape(-1),
                                       w.scales.numpy().reshape(-1), M, K, nl, 128, 16)
        words, scales = P.gather_columns(torch.from_numpy(O.pack(codes, 16)),
                                         torch.from_numpy(cs), M, WORLD,
                                         widths=[e - s for s, e in w.shards], bits=16,
                                         block=128)
        if rank == 0:
            result_q.put((words.numpy(), scales.numpy()))
    finally:
        dist.destroy_process_group()


def test_sharded_qgemm_uneven_shards():
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_qgemm_uneven_rank, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    words, scales = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    a, b = _inputs(M=32, K=256, N=640)
    M, K = a.shape
    N = b.shape[1]
    pa, sa, _ = O.quantize(a.numpy(), 8, "int", 128)
    pb, sb, _ = O.quantize(b.numpy(), 8, "int", 128)
    codes, cs, _ = O.qscale_matmul(O.unpack(pa, 8, M * K), sa, O.unpack(pb, 8, K * N), sb,
                                   M, K, N, 128, 16)
    assert np.array_equal(words, O.pack(codes, 16))
    assert np.array_equal(scales.view(np.uint32), cs.view(np.uint32))


# ── Kronecker split of the h unrotation over column shards ──

def _cross_stage(t, signs):
    """numpy stand-in for mxb_hadamard_cross: t [G, M, L] -> [M, G*L]."""
    G = t.shape[0]
    v = [t[g].astype(np.float32) for g in range(G)]
    h = G // 2
    while h >= 1:
        for g in range(G):
            if g & h:
                continue
            e, o = v[g], v[g + h]
            v[g], v[g + h] = (e + o).astype(np.float32), (e - o).astype(np.float32)
        h //= 2
    z = np.concatenate([(vg / np.float32(np.sqrt(G))).astype(np.float32) for vg in v], axis=1)
    return (z * signs[None, :]).astype(np.float32)


def _kron_rank(rank, port, world, result_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from qtpytorch_b200.dtypes import get_mx_dtype
        from qtpytorch_b200.hadamard import sign_vector
        dt = get_mx_dtype("int4dh")
        M, N = 5, 1024
        y = np.random.default_rng(5).standard_normal((M, N)).astype(np.float32)
        L = N // world
        # this rank's local stage: the plain normalized WHT of its columns
        t = torch.from_numpy(O.fwht(y[:, rank * L:(rank + 1) * L]))
        g = P._all_gather(t.contiguous(), world, None)  # [G, M, L], as NCCL lays it out
        z = _cross_stage(g.numpy(), sign_vector(N, dt.hadamard_seed).numpy())
        if rank == 0:
            result_q.put(z)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_kronecker_split_unrotation(world):
    """Local L-point transforms + one gather + the G-point stage equal the
    full-row unrotation (mxtorch.py:2892-2904) to fp32 rounding."""
    from qtpytorch_b200.dtypes import get_mx_dtype
    from qtpytorch_b200.hadamard import sign_vector
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_kron_rank, args=(r, port, world, q)) for r in range(world)]
    for p in procs:
        p.start()
    z = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    y = np.random.default_rng(5).standard_normal((5, 1024)).astype(np.float32)
    ref = O.unrotate(y, sign_vector(1024, get_mx_dtype("int4dh").hadamard_seed).numpy())
    bound = np.abs(y).astype(np.float64).sum(axis=1, keepdims=True) / np.sqrt(1024)
    assert np.all(np.abs(z.astype(np.float64) - ref) <= 1e-6 * bound)


@pytest.mark.parametrize("shape,block,world", [((12, 256), 128, 3), ((7, 96), 64, 2),
                                               ((5, 100), 128, 2), ((300,), 64, 2)])
def test_h_row_sharded_quantize_concatenates_to_full(shape, block, world):
    """Row-sharded quantize of an h dtype: whole rows per rank (rotation is per
    row), shard starts on block boundaries; concatenation = full quantize."""
    from qtpytorch_b200.dtypes import get_mx_dtype
    from qtpytorch_b200.hadamard import sign_vector
    dt = get_mx_dtype("int4dh")
    x = np.random.default_rng(9).standard_normal(shape).astype(np.float32)
    d = shape[-1] if len(shape) >= 2 else x.size
    signs = sign_vector(d, dt.hadamard_seed).numpy()
    full_p, full_s, _ = O.quantize(x, 4, "int", block, True, signs)
    rows = x.reshape(-1, d)
    ps, ss, got_rows = [], [], 0
    for r in range(world):
        r0, r1 = P.h_row_range(shape, block, 4, world, r)
        assert r0 == got_rows
        got_rows = r1
        if r1 > r0:
            part = rows[r0:r1] if len(shape) >= 2 else rows[r0:r1].reshape(-1)
            p, s, _ = O.quantize(part, 4, "int", block, True, signs)
            ps.append(p)
            ss.append(s)
    assert got_rows == rows.shape[0]
    assert np.array_equal(np.concatenate(ps), full_p)
    assert np.array_equal(np.concatenate(ss), full_s)
