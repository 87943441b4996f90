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


@pytest.mark.gpu
@pytest.mark.parametrize("M,K,N,dt,x_dt,block", [
    (64, 512, 256, "int4d", torch.bfloat16, 128),    # tcgen05, K-major codes
    (300, 1024, 384, "int8d", torch.bfloat16, 64),   # tcgen05, ragged M tile
    (40, 256, 128, "int2d", torch.bfloat16, 128),    # tcgen05, 2-bit
    (48, 512, 256, "float4d", torch.bfloat16, 128),  # tcgen05, grid codes
    (7, 384, 96, "int4d", torch.float32, 128),       # CUDA-core kernel
    (33, 200, 72, "int1d", torch.bfloat16, 8),       # CUDA-core: 1-bit, blocks across rows
    (5, 256, 64, "int4dh", torch.float32, 128),      # h weight: rotated x
])
def test_linear_wonly_kmajor(M, K, N, dt, x_dt, block):
    """y = x @ dequant(W)^T for W [N, K] quantized flat along K, without a
    dequantized weight (mx_dynamic_linear's matmul, mxtorch.py:8947-8978)."""
    from qtpytorch_b200 import dynamic as D
    d = mxb.get_mx_dtype(dt)
    g = torch.Generator().manual_seed(M * 7 + K)
    w = torch.randn(N, K, generator=g) * 0.02
    x = torch.randn(M, K, generator=g).to(x_dt)
    q = mxb.mx_tensor.quantize(w.cuda(), d, block)
    n0 = mxb._lib.load().mxb_launch_count()
    y = D._kmajor_linear(x.cuda(), q, K, N).cpu().numpy().astype(np.float64)
    assert mxb._lib.load().mxb_launch_count() > n0
    assert mxb._lib.load().mxb_device_error(1) == 0
    w_dq = q.dequantize().cpu().numpy().reshape(N, K).astype(np.float64)
    xf = x.float().numpy().astype(np.float64)
    ref, mag = xf @ w_dq.T, np.abs(xf) @ np.abs(w_dq).T
    if d.is_hadamard:  # rotation error of x enters through |rotate(x)| @ |D|
        D_rot = mxb.ops.dequantize(q._mx_packed, q._mx_scales, d.base, q._mx_n, block,
                                   (N, K)).cpu().numpy().astype(np.float64)
        xr = mxb.ops.hadamard_rows(x.float().cuda(), d.hadamard_seed, False).cpu().numpy()
        mag = np.abs(xr.astype(np.float64)) @ np.abs(D_rot).T
    assert np.all(np.abs(y - ref) <= LIN_TOL * mag + 1e-30), float(np.max(np.abs(y - ref) / mag))


@pytest.mark.gpu
def test_mx_dynamic_linear_prefill_bf16():
    """bf16 tokens at a prefill size go to the tcgen05 K-major kernel."""
    lin = torch.nn.Linear(512, 384, bias=True)
    g = torch.Generator().manual_seed(77)
    with torch.no_grad():
        lin.weight.copy_(torch.randn(384, 512, generator=g) * 0.02)
        lin.bias.copy_(torch.randn(384, generator=g) * 0.1)
    m = mxb.mx_dynamic_linear.from_linear(lin, "int4d", "int8d")
    x = torch.randn(2, 96, 512, generator=g).bfloat16()
    out = m(x.cuda()).cpu().numpy().astype(np.float64)
    w_dq = m.weight.dequantize().cpu().numpy().reshape(384, 512).astype(np.float64)
    xf = x.float().numpy().reshape(-1, 512).astype(np.float64)
    b = lin.bias.detach().numpy().astype(np.float64)
    ref = (xf @ w_dq.T + b).reshape(2, 96, 384)
    mag = (np.abs(xf) @ np.abs(w_dq).T + np.abs(b)).reshape(2, 96, 384)
    assert np.all(np.abs(out - ref) <= LIN_TOL * mag)


@pytest.mark.gpu
def test_fused_int8_linear_mixed_operands():
    """Operands the integer GEMM does not take (int8 x against an int4 weight)
    run as dequant(x) against the packed weight on the K-major kernel."""
    g = torch.Generator().manual_seed(78)
    x = torch.randn(9, 256, generator=g)
    w = torch.randn(64, 256, generator=g) * 0.02
    xq = mxb.mx_tensor.quantize(x.cuda(), mxb.get_mx_dtype("int8d"), 128)
    wq = mxb.mx_tensor.quantize(w.cuda(), mxb.get_mx_dtype("int4d"), 128)
    out = mxb.fused_int8_linear(xq, wq).cpu().numpy().astype(np.float64)
    x_dq = xq.dequantize().cpu().numpy().astype(np.float64)
    w_dq = wq.dequantize().cpu().numpy().reshape(64, 256).astype(np.float64)
    ref, mag = x_dq @ w_dq.T, np.abs(x_dq) @ np.abs(w_dq).T
    assert np.all(np.abs(out - ref) <= LIN_TOL * mag)
