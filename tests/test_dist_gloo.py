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
