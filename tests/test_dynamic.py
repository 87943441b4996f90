"""dynamic_quantize / fused_int8_linear / mx_dynamic_linear
(mxtorch.py:2665-2712, 3910-3960, 8870-8978).

CPU: the oracle against fixtures made by running the reference
(tests/golden/make_golden_dynamic.py).  GPU: the CUDA path against the same
fixtures and the oracle: dynamic_quantize bit-exact (codes, scales,
dequantized values); the linears within 1e-5 of |x| @ |W|^T (+ |bias|) of
the float64 product of the dequantized operands.
"""
import numpy as np
import pytest
import torch

import make_golden_dynamic as GD
import qtpytorch_b200 as mxb
from oracle import mx_oracle as O

BITS = {"int8d": 8, "int4d": 4, "int2d": 2}
LIN_TOL = 1e-5


def _u32(a):
    return np.ascontiguousarray(a).view(np.uint32)


@pytest.mark.parametrize("c", GD.DYN_CASES, ids=lambda c: c[0])
def test_oracle_dynamic_quantize_matches_reference(golden_dynamic, c):
    key, dt, gran, _, _, _, block = c
    x = GD.make_dyn_input(c).float().numpy()
    p, s, b, n = O.dynamic_quantize(x, BITS[dt], gran, block)
    g = golden_dynamic
    assert np.array_equal(p.view(np.int8), g[f"{key}/packed"].view(np.int8))
    assert np.array_equal(_u32(s), _u32(g[f"{key}/scales"]))
    assert b == int(g[f"{key}/block"]) and n == int(g[f"{key}/n"])
    dq = O.dequant_flat(p, s, BITS[dt], "int", n, b)
    assert np.array_equal(_u32(np.asarray(dq, np.float32).reshape(-1)),
                          _u32(g[f"{key}/dequant"].reshape(-1)))


def _oracle_fused(c):
    key, M, K, N, gran, wblock, _, _ = c
    x, w, b = GD.make_fused_inputs(c)
    if gran == "per_token":
        xp, xs, xb, xn = O.dynamic_quantize(x.numpy(), 8, "per_token")
    else:
        xp, xs, xn = O.quantize(x.numpy(), 8, "int", 128)
        xb = 128
    wp, ws, wn = O.quantize(w.numpy(), 8, "int", wblock)
    x_dq = np.asarray(O.dequant_flat(xp, xs, 8, "int", xn, xb), np.float32).reshape(M, K)
    w_dq = np.asarray(O.dequant_flat(wp, ws, 8, "int", wn, wblock), np.float32).reshape(N, K)
    bias = None if b is None else b.numpy()
    ref = O.fused_int8_linear_ref64(x_dq, w_dq, bias)
    mag = np.abs(x_dq).astype(np.float64) @ np.abs(w_dq).astype(np.float64).T
    if bias is not None:
        mag = mag + np.abs(bias)[None, :]
    return ref, mag


@pytest.mark.parametrize("c", GD.FUSED_CASES, ids=lambda c: c[0])
def test_oracle_fused_int8_linear_matches_reference(golden_dynamic, c):
    ref, mag = _oracle_fused(c)
    out = golden_dynamic[f"{c[0]}/out"].astype(np.float64)
    assert np.all(np.abs(out - ref) <= LIN_TOL * mag)


@pytest.mark.gpu
@pytest.mark.parametrize("c", GD.DYN_CASES, ids=lambda c: c[0])
def test_dynamic_quantize_bit_exact(golden_dynamic, c):
    key, dt, gran, shape, _, _, block = c
    q = mxb.dynamic_quantize(GD.make_dyn_input(c).cuda(), dt, gran, block)
    g = golden_dynamic
    assert q._mx_block == int(g[f"{key}/block"]) and q._mx_n == int(g[f"{key}/n"])
    assert tuple(q._mx_orig_shape) == tuple(shape)
    assert np.array_equal(q._mx_packed.cpu().numpy().view(np.int8), g[f"{key}/packed"].view(np.int8))
    assert np.array_equal(_u32(q._mx_scales.cpu().numpy()), _u32(g[f"{key}/scales"]))
    dq = q.dequantize().cpu().numpy().reshape(-1)
    assert np.array_equal(_u32(dq), _u32(g[f"{key}/dequant"].reshape(-1)))


@pytest.mark.gpu
@pytest.mark.parametrize("n,K", [(4096 * 16, 4096), (3 * 11008, 11008), (5 * 96, 96)])
def test_dynamic_quantize_per_token_large(n, K):
    # blocks above 256 take the two-pass kernel; compare with the oracle
    x = torch.randn(n, generator=torch.Generator().manual_seed(K)).view(-1, K) * 3
    q = mxb.dynamic_quantize(x.cuda(), "int8d", "per_token")
    p, s, b, _ = O.dynamic_quantize(x.numpy(), 8, "per_token")
    assert q._mx_block == b == K
    assert np.array_equal(q._mx_packed.cpu().numpy().view(np.int8), p.view(np.int8))
    assert np.array_equal(_u32(q._mx_scales.cpu().numpy()), _u32(s))


@pytest.mark.gpu
@pytest.mark.parametrize("c", GD.FUSED_CASES, ids=lambda c: c[0])
def test_fused_int8_linear(golden_dynamic, c):
    key, M, K, N, gran, wblock, _, _ = c
    x, w, b = GD.make_fused_inputs(c)
    if gran == "per_token":
        xq = mxb.dynamic_quantize(x.cuda(), "int8d", "per_token")
    else:
        xq = mxb.mx_tensor.quantize(x.cuda(), mxb.get_mx_dtype("int8d"), 128)
    wq = mxb.mx_tensor.quantize(w.cuda(), mxb.get_mx_dtype("int8d"), wblock)
    n0 = mxb._lib.load().mxb_launch_count()
    out = mxb.fused_int8_linear(xq, wq, None if b is None else b.cuda(), wblock)
    assert mxb._lib.load().mxb_launch_count() > n0  # the packed GEMM ran
    assert out.shape == (M, N) and out.dtype == torch.float32
    ref, mag = _oracle_fused(c)
    got = out.cpu().numpy().astype(np.float64)
    assert np.all(np.abs(got - ref) <= LIN_TOL * mag)
    gold = golden_dynamic[f"{key}/out"].astype(np.float64)
    assert np.all(np.abs(got - gold) <= 2 * LIN_TOL * mag)


@pytest.mark.gpu
@pytest.mark.parametrize("c", GD.DLIN_CASES, ids=lambda c: c[0])
def test_mx_dynamic_linear(golden_dynamic, c):
    key, T, K, N, wdt, has_bias, _ = c
    lin, x = GD.make_dlin_inputs(c)
    m = mxb.mx_dynamic_linear.from_linear(lin, wdt, "int8d")
    g = golden_dynamic
    assert np.array_equal(m.weight._mx_packed.cpu().numpy().view(np.int8),
                          g[f"{key}/w_packed"].view(np.int8))
    assert np.array_equal(_u32(m.weight._mx_scales.cpu().numpy()), _u32(g[f"{key}/w_scales"]))
    out = m(x.cuda()).cpu().numpy().astype(np.float64)
    w_dq = m.weight.dequantize().cpu().numpy().reshape(N, K).astype(np.float64)
    xf = x.numpy().astype(np.float64)
    mag = np.abs(xf) @ np.abs(w_dq).T
    ref = xf @ w_dq.T
    if has_bias:
        ref = ref + lin.bias.detach().numpy()[None, :]
        mag = mag + np.abs(lin.bias.detach().numpy())[None, :]
    assert np.all(np.abs(out - ref) <= LIN_TOL * mag)
    assert np.all(np.abs(out - g[f"{key}/out"]) <= 2 * LIN_TOL * mag)
