"""Parity at the full sizes the benchmark runs.

* the int4dh weight-only linear, W 8192 x 8192 ~ N(0, 0.02) with
  8 outlier input channels x25, x bf16 [4096, 8192].  The packed codes and
  scales of W^T are compared bit for bit with the oracle's (8192-point row
  WHT, mxtorch.py:1720-1736, 2866-2890), and sampled output columns with
  y64 = x @ unrotate(dequant(W^T)) in float64 (mxtorch.py:7454-7473,
  2892-2904).  The unrotation mixes every column of a row, so the
  per-element bound propagates |x| @ |dequant| through |H| / sqrt(n):
  |y - y64| <= 1e-5 * rowsum(|x| @ |D|) / sqrt(n), plus a norm-relative
  1e-5 over the sampled columns.
* configs[4] at 2^28 elements (fp32 and bf16 N(0,1), and a Student-t nu=3
  tail): quantize and dequantize of int2d / int1d / float4d, blocks 32 and
  128, checked bit for bit against the oracle on 2^16 random blocks plus the
  first and the last block (blocks are independent).
* the int GEMM's int32 K-block partials P_kb = A[:, kb] @ B[kb, :]
  (mxtorch.py:1357-1370): with unit scales and one K-block the kernel's fp32
  C is P_kb itself (|P| < 2^24 is exact in fp32), compared with the oracle's
  integer products for every K-block, on the tcgen05 and the CUDA-core
  kernels.
"""
import math

import numpy as np
import pytest
import torch

import qtpytorch_b200 as mxb
from oracle import mx_oracle as O
from qtpytorch_b200 import _lib as L
from qtpytorch_b200 import ops

pytestmark = pytest.mark.gpu

LIN_TOL = 1e-5


def _u32(a):
    return np.ascontiguousarray(a).view(np.uint32)


# ── configs[3] ───────────────────────────────────────────────────────────────
@pytest.fixture(scope="module")
def int4dh_8192():
    g3 = torch.Generator().manual_seed(3)
    W = torch.randn(8192, 8192, generator=g3) * 0.02
    W[:, torch.randperm(8192, generator=g3)[:8]] *= 25.0
    lin = torch.nn.Linear(8192, 8192, bias=False)
    with torch.no_grad():
        lin.weight.copy_(W)
    dt = mxb.get_mx_dtype("int4dh")
    ml = mxb.mx_linear.from_linear(lin.cuda(), dt, 128)
    return ml, W, dt


def test_config4_int4dh_codes_bit_exact(int4dh_8192):
    ml, W, dt = int4dh_8192
    wt = W.t().contiguous().numpy()
    signs = mxb.sign_vector(8192, dt.hadamard_seed).numpy()
    p, s, n = O.quantize(wt, 4, "int", 128, hadamard=True, signs=signs)
    q = ml._mx_weight
    assert q._mx_n == n
    assert np.array_equal(_u32(q._mx_scales.cpu().numpy()), _u32(s))
    assert np.array_equal(q._mx_packed.cpu().numpy(), p)


def _hadamard_cols(n, cols):
    """Columns `cols` of the Sylvester Hadamard matrix H_n (entries +-1):
    H[i, j] = (-1)^popcount(i & j)."""
    i = np.arange(n, dtype=np.int64)[:, None]
    j = np.asarray(cols, dtype=np.int64)[None, :]
    v = i & j
    par = np.zeros_like(v)
    while np.any(v):
        par ^= v & 1
        v >>= 1
    return (1 - 2 * par).astype(np.float64)


@pytest.mark.parametrize("mode", ["module", "sharded_g1"])
def test_config4_linear_full_size(int4dh_8192, mode):
    ml, _W, dt = int4dh_8192
    x = torch.randn(4096, 8192, generator=torch.Generator().manual_seed(4)).bfloat16().cuda()
    if mode == "module":
        y = ml(x)
    else:
        from qtpytorch_b200 import parallel as P
        y = P.sharded_linear(x, P.ShardedLinearWeight.from_module(ml, 1, 0))
    assert L.load().mxb_device_error(1) == 0
    n = 8192
    cols = np.sort(np.random.default_rng(44).choice(n, 62, replace=False))
    cols = np.concatenate([[0], cols, [n - 1]])
    q = ml._mx_weight
    # rotated-domain dequantized W^T [K, N]: the base dtype's dequantize (the
    # mx_tensor's own dequantize would also unrotate)
    D = ops.dequantize(q._mx_packed, q._mx_scales, dt.base, q._mx_n, q._mx_block,
                       q._mx_orig_shape).double()
    x64 = x.double()
    signs = mxb.sign_vector(n, dt.hadamard_seed).double().cuda()
    Hc = torch.from_numpy(_hadamard_cols(n, cols)).cuda()
    # unrotate(row) = WHT(row) / sqrt(n) * signs, restricted to `cols`
    weff = (D @ Hc) / math.sqrt(n) * signs[cols]
    ref = (x64 @ weff).cpu().numpy()
    bound = ((x64.abs() @ D.abs()).sum(dim=1, keepdim=True) / math.sqrt(n)).cpu().numpy()
    got = y[:, torch.from_numpy(cols).cuda()].double().cpu().numpy()
    err = np.abs(got - ref)
    assert np.all(err <= LIN_TOL * bound), float((err / bound).max())
    rel = np.linalg.norm(got - ref) / np.linalg.norm(ref)
    assert rel <= LIN_TOL, rel


# ── configs[4] at 2^28 ───────────────────────────────────────────────────────
def _sample_blocks(nb, k, seed):
    idx = np.random.default_rng(seed).choice(nb - 2, k, replace=False) + 1
    return np.concatenate([[0], np.sort(idx), [nb - 1]])


def _packed_rows(packed, block, bits, idx):
    per = block * bits // 8  # bytes of one block (block * bits is a multiple of 8 here)
    t = packed.view(torch.uint8)[: (packed.numel() // per) * per].view(-1, per)
    return t[torch.from_numpy(idx).cuda()].cpu().numpy().view(np.int8).reshape(-1)


@pytest.mark.parametrize("dist", ["normal", "student_t"])
@pytest.mark.parametrize("in_dt", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("dt", ["int2d", "int1d", "float4d"])
@pytest.mark.parametrize("block", [32, 128])
def test_sweep_2e28_sampled_blocks(dt, block, in_dt, dist):
    n = 1 << 28
    torch.cuda.manual_seed(5)
    if dist == "normal":
        x = torch.randn(n, device="cuda")
    else:
        x = torch.distributions.StudentT(torch.tensor(3.0, device="cuda")).sample((n,))
    x = x.to(in_dt)
    d = mxb.get_mx_dtype(dt)
    q = mxb.mx_tensor.quantize(x, d, block)
    nb = n // block
    idx = _sample_blocks(nb, 1 << 16, block + d.bits)
    idx_t = torch.from_numpy(idx).cuda()
    xs = x.view(nb, block)[idx_t].float().cpu().numpy()
    p_ref, s_ref, _ = O.quantize(xs.reshape(-1), d.bits, d.kind, block)
    assert np.array_equal(_u32(q._mx_scales[idx_t].cpu().numpy()), _u32(s_ref))
    assert np.array_equal(_packed_rows(q._mx_packed, block, d.bits, idx), p_ref)
    dq = ops.dequantize(q._mx_packed, q._mx_scales, d, n, block)
    ref = O.dequant_flat(p_ref, s_ref, d.bits, d.kind, xs.size, block)
    got = dq.view(nb, block)[idx_t].cpu().numpy().reshape(-1)
    assert np.array_equal(_u32(got), _u32(ref))
    del x, q, dq
    torch.cuda.empty_cache()


# ── int32 K-block partials ───────────────────────────────────────────────────
@pytest.mark.parametrize("M,K,N,dt", [(256, 1024, 384, "int8d"), (128, 512, 256, "int4d"),
                                      (96, 384, 200, "int8d"), (64, 256, 72, "int2d")])
def test_kblock_partials_bit_exact(M, K, N, dt):
    """Each K-block's exact integer partial through the kernel: A[:, kb] and
    B[kb, :] with unit scales, so C = P_kb."""
    d = mxb.get_mx_dtype(dt)
    g = torch.Generator().manual_seed(M + K + N)
    a = torch.randn(M, K, generator=g)
    b = torch.randn(K, N, generator=g)
    pa, _, _ = O.quantize(a.numpy(), d.bits, "int", 128)
    pb, _, _ = O.quantize(b.numpy(), d.bits, "int", 128)
    ca = O.unpack(pa, d.bits, M * K).reshape(M, K)
    cb = O.unpack(pb, d.bits, K * N).reshape(K, N)
    ref = O.kblock_partials(ca.reshape(-1), cb.reshape(-1), M, K, N, 128)
    for kb in range(K // 128):
        sa = np.ascontiguousarray(ca[:, kb * 128:(kb + 1) * 128])
        sb = np.ascontiguousarray(cb[kb * 128:(kb + 1) * 128, :])
        ap = torch.from_numpy(O.pack(sa.reshape(-1), d.bits)).cuda()
        bp = torch.from_numpy(O.pack(sb.reshape(-1), d.bits)).cuda()
        ones_a = torch.ones(-(-M * 128 // 128), device="cuda")
        ones_b = torch.ones(N, device="cuda")  # [K/block = 1, N]
        _, _, c = ops.qgemm(ap, ones_a, bp, ones_b, M, 128, N, d.bits, 128, 32)
        assert L.load().mxb_device_error(1) == 0
        got = c.cpu().numpy()
        assert np.all(got == np.round(got))
        assert np.array_equal(got.astype(np.int64), ref[kb].astype(np.int64)), kb
