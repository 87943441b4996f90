"""Multi-GPU tests (run where the box has two or more GPUs; skipped
otherwise): the column-sharded matmul with the output gather fused into
the tcgen05 kernel, launched as one process per GPU with torchrun."""
import os
import socket
import subprocess
import sys

import numpy as np
import pytest
import torch

import qtpytorch_b200 as mxb
from qtpytorch_b200 import parallel as P

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def test_fused_gather_single_rank_equals_plain_matmul():
    """World 1: the fused-output entry writes the same int16d result as the
    plain matmul (its output list holds only this rank's buffers)."""
    g = torch.Generator().manual_seed(3)
    a = torch.randn(256, 384, generator=g).cuda()
    b = torch.randn(384, 512, generator=g).cuda()
    qa = mxb.mx_tensor.quantize(a, mxb.int8d, 128)
    qb = mxb.mx_tensor.quantize(b, mxb.int8d, 128)
    w = P.ShardedQGemmWeight(qb, 1, 0)
    peers = P.PeerOutputs(256, 512, 128, 1, 0)
    c = P.sharded_qgemm_fused(qa, w, peers)
    ref = qa @ qb
    assert torch.equal(c._mx_packed, ref._mx_packed.view(torch.int32))
    assert torch.equal(c._mx_scales, ref._mx_scales)


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_fused_gather_two_ranks():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr", "127.0.0.1", "--master-port", str(_port()),
           os.path.join(HERE, "dist_fused_worker.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    assert "OK" in r.stdout


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_sharded_h_linear_and_quantize_two_ranks():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr", "127.0.0.1", "--master-port", str(_port()),
           os.path.join(HERE, "dist_linear_worker.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    assert "OK" in r.stdout


@pytest.mark.parametrize("N", [1024, 8192])
def test_kron_split_single_rank(N):
    """G = 1 of the split: the local transform of all N columns (unit signs)
    and the sign stage (mxb_hadamard_cross) do the module's full-row
    unrotation's arithmetic in the same order, so the results are identical;
    sharded_linear itself skips the split at world 1."""
    dt = mxb.get_mx_dtype("int4dh")
    g = torch.Generator().manual_seed(N)
    lin = torch.nn.Linear(512, N, bias=False)
    with torch.no_grad():
        lin.weight.copy_(torch.randn(N, 512, generator=g) * 0.02)
    ml = mxb.mx_linear.from_linear(lin.cuda(), dt, 128)
    x = torch.randn(48, 512, generator=g).bfloat16().cuda()
    sw = P.ShardedLinearWeight.from_module(ml, 1, 0)
    assert sw.kron_split
    from qtpytorch_b200 import ops
    y0 = ops.linear_wonly(x, sw.codes, sw.scales, 512, N, dt, 128)
    t = ops.hadamard_rows(y0, None, inverse=True)
    y = ops.hadamard_cross(t, 48, N, 1, dt.hadamard_seed)
    ref = ml(x)
    assert torch.equal(y, ref)
    assert torch.equal(P.sharded_linear(x, sw), ref)
