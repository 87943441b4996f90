"""fused_linear_relu / fused_silu_and_mul (mxtorch.py:4012-4074, 4077-4109).

Fixtures come from running the reference's CPU branches
(tests/golden/make_golden_dynamic.py).  fused_linear_relu is bit-exact (the
packed matmul, dequantize, relu and the fp32 bias add are each exact
restatements).  fused_silu_and_mul: within 4e-7 * |silu(g) * u| + 1e-30 of
the float64 formula on the dequantized operands (fp32 exp, divide and
multiply), and within twice that of the reference's own fp32 output.
"""
import numpy as np
import pytest
import torch

import make_golden_dynamic as GD
import qtpytorch_b200 as mxb
from oracle import mx_oracle as O

SILU_TOL = 4e-7


def _u32(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def _silu_ref64(c):
    _, dt, shape, block, _ = c
    g, u = GD.make_silu_inputs(c)
    d = mxb.get_mx_dtype(dt)
    gp, gs, gn = O.quantize(g.numpy(), d.bits, d.kind, block)
    up, us, un = O.quantize(u.numpy(), d.bits, d.kind, block)
    gd = np.asarray(O.dequant_flat(gp, gs, d.bits, d.kind, gn, block), np.float64).reshape(shape)
    ud = np.asarray(O.dequant_flat(up, us, d.bits, d.kind, un, block), np.float64).reshape(shape)
    return gd / (1.0 + np.exp(-gd)) * ud


@pytest.mark.parametrize("c", GD.SILU_CASES, ids=lambda c: c[0])
def test_oracle_silu_formula_matches_reference(golden_dynamic, c):
    ref = _silu_ref64(c)
    gold = golden_dynamic[f"{c[0]}/out"].astype(np.float64)
    assert np.all(np.abs(gold - ref) <= SILU_TOL * np.abs(ref) + 1e-30)


@pytest.mark.gpu
@pytest.mark.parametrize("c", GD.RELU_CASES, ids=lambda c: c[0])
def test_fused_linear_relu_bit_exact(golden_dynamic, c):
    key, _, _, N, dt, _, w_mx, _ = c
    x, w, b = GD.make_relu_inputs(c)
    d = mxb.get_mx_dtype(dt)
    b_d = None if b is None else b.cuda()
    if w_mx:
        y = mxb.fused_linear_relu(x.cuda(), mxb.mx_tensor.quantize(w.t().cuda(), d, 128), b_d, 128)
    else:
        y = mxb.fused_linear_relu(x.cuda(), w.cuda(), b_d, 128, d)
    gold = golden_dynamic[f"{key}/out"]
    assert tuple(y.shape) == gold.shape
    assert np.array_equal(_u32(y.cpu().numpy()), _u32(gold))


@pytest.mark.gpu
@pytest.mark.parametrize("c", GD.SILU_CASES, ids=lambda c: c[0])
def test_fused_silu_and_mul(golden_dynamic, c):
    key, dt, shape, block, _ = c
    g, u = GD.make_silu_inputs(c)
    d = mxb.get_mx_dtype(dt)
    gq = mxb.mx_tensor.quantize(g.cuda(), d, block)
    uq = mxb.mx_tensor.quantize(u.cuda(), d, block)
    n0 = mxb._lib.load().mxb_launch_count()
    y = mxb.fused_silu_and_mul(gq, uq)
    assert mxb._lib.load().mxb_launch_count() == n0 + 1  # one fused kernel
    assert tuple(y.shape) == tuple(shape)
    got = y.cpu().numpy().astype(np.float64)
    ref = _silu_ref64(c)
    assert np.all(np.abs(got - ref) <= SILU_TOL * np.abs(ref) + 1e-30)
    gold = golden_dynamic[f"{key}/out"].astype(np.float64)
    assert np.all(np.abs(got - gold) <= 2 * SILU_TOL * np.abs(ref) + 1e-30)


@pytest.mark.gpu
@pytest.mark.parametrize("dt", ["int8d", "int4d", "int1d", "float4d"])
@pytest.mark.parametrize("n,block", [(1 << 20, 128), (1000, 8), (777, 7)])
def test_dequantize_relu_equals_relu_of_dequantize(dt, n, block):
    # aligned warp-chunk kernel, ragged tail, and the per-element kernel (block 7)
    d = mxb.get_mx_dtype(dt)
    x = torch.randn(n, generator=torch.Generator().manual_seed(n)).cuda()
    q = mxb.mx_tensor.quantize(x, d, block)
    from qtpytorch_b200 import ops
    got = ops.dequantize_relu(q._mx_packed, q._mx_scales, d, n, block).cpu().numpy()
    ref = np.maximum(q.dequantize().cpu().numpy(), np.float32(0))
    assert np.array_equal(_u32(got), _u32(ref))
