"""The CPU oracle reproduces the reference's own outputs bit for bit."""
import numpy as np
import pytest
import torch

import cases
from oracle import mx_oracle as O
from qtpytorch_b200.dtypes import get_mx_dtype
from qtpytorch_b200.hadamard import sign_vector


def _np(x):
    return x.float().numpy() if isinstance(x, torch.Tensor) else np.asarray(x)


def test_pack_known_answers(golden):
    # mxtorch_test.py:86-93: round trip of [3,-2,7,-8,0,1,-1,4] at 4 bits
    v4 = np.array([3, -2, 7, -8, 0, 1, -1, 4])
    assert np.array_equal(O.pack(v4, 4), golden["kat_pack4"])
    assert np.array_equal(O.unpack(golden["kat_pack4"], 4, 8), v4)
    v2 = np.array([1, -2, 0, -1, 1, -2, 0, 1])
    assert np.array_equal(O.pack(v2, 2), golden["kat_pack2"])
    assert np.array_equal(O.unpack(golden["kat_pack2"], 2, 8), v2)
    v1 = np.array([0, 1, 0, 1, 1, 0, 1, 0])
    assert np.array_equal(O.pack(v1, 1), golden["kat_pack1"])


def test_pack16_roundtrip():
    v = np.array([-32767, 32767, 0, -1, 5, -5, 123], np.int32)
    assert np.array_equal(O.unpack(O.pack(v, 16), 16, v.size), v)


@pytest.mark.parametrize("c", cases.QUANT_CASES, ids=lambda c: c["key"])
def test_quantize_matches_reference(golden, c):
    dt = get_mx_dtype(c["dtype"])
    x = _np(cases.make_input(c))
    k = c["key"]
    signs = None
    if dt.is_hadamard:
        d = x.shape[-1] if x.ndim >= 2 else x.size
        signs = sign_vector(d, dt.hadamard_seed).numpy()
        assert np.array_equal(signs, golden[f"{k}/signs"])
        assert int(golden[f"{k}/seed"]) == dt.hadamard_seed
        if f"{k}/rotated" in golden:
            xr = x if x.ndim >= 2 else x.reshape(1, -1)
            assert np.array_equal(O.rotate(xr, signs), golden[f"{k}/rotated"])
    packed, scales, n = O.quantize(x, dt.bits, dt.kind, c["block"], dt.is_hadamard, signs)
    assert n == int(golden[f"{k}/n"])
    assert np.array_equal(scales.view(np.uint32), golden[f"{k}/scales"].view(np.uint32))
    assert np.array_equal(packed, golden[f"{k}/packed"])
    if f"{k}/dequant" in golden:
        dq = O.dequantize(packed, scales, dt.bits, dt.kind, x.shape, c["block"],
                          dt.is_hadamard, signs)
        ref = golden[f"{k}/dequant"]
        assert np.array_equal(dq.view(np.uint32), ref.view(np.uint32))


def test_h_dequant_1d_equals_reference_literal(golden):
    # for 1-D tensors the reference's own dequantize is the contract too
    k = "h_int2dh_1d300"
    assert np.array_equal(golden[f"{k}/dequant"], golden[f"{k}/dequant_ref_literal"])


@pytest.mark.parametrize("c", cases.GEMM_CASES, ids=lambda c: c["key"])
def test_qscale_matmul_matches_reference(golden, c):
    dt = get_mx_dtype(c["dtype"])
    dtb = get_mx_dtype(c.get("dtype_b", c["dtype"]))
    a, b = cases.make_gemm_inputs(c)
    M, K, N, blk = c["M"], c["K"], c["N"], c["block"]

    def q(x, d):
        signs = None
        if d.is_hadamard:
            signs = sign_vector(x.shape[-1], d.hadamard_seed).numpy()
        return O.quantize(_np(x), d.bits, d.kind, blk, hadamard=d.is_hadamard, signs=signs)

    pa, sa, _ = q(a, dt)
    pb, sb, _ = q(b, dtb)
    ca = O.unpack(pa, dt.bits, M * K)
    cb = O.unpack(pb, dt.bits, K * N)
    out_bits = int(golden[f"{c['key']}/c_bits"])
    codes, cs, _C = O.qscale_matmul(ca, sa, cb, sb, M, K, N, blk, out_bits)
    assert np.array_equal(cs.view(np.uint32), golden[f"{c['key']}/c_scales"].view(np.uint32))
    assert np.array_equal(O.pack(codes, out_bits), golden[f"{c['key']}/c_packed"])
    assert int(golden[f"{c['key']}/c_block"]) == blk


@pytest.mark.parametrize("c", cases.LINEAR_CASES, ids=lambda c: c["key"])
def test_linear_matches_reference(golden, c):
    dt = get_mx_dtype(c["dtype"])
    lin, x = cases.make_linear_inputs(c)
    wt = lin.weight.data.t().contiguous().numpy()
    pw, sw, _ = O.quantize(wt, dt.bits, dt.kind, c["block"])
    assert np.array_equal(pw, golden[f"{c['key']}/w_packed"])
    assert np.array_equal(sw, golden[f"{c['key']}/w_scales"])
    wdq = O.dequantize(pw, sw, dt.bits, dt.kind, wt.shape, c["block"])
    y64, bound = O.linear_ref64(_np(x), wdq)
    y = golden[f"{c['key']}/y"].astype(np.float64)
    assert np.all(np.abs(y - y64) <= 1e-5 * bound + 1e-30)


def test_wht_matches_reference(golden):
    g = torch.Generator().manual_seed(11)
    xw = torch.randn(2, 1024, generator=g).numpy()
    assert np.array_equal(O.fwht(xw), golden["wht/y"])


@pytest.mark.parametrize("c", [c for c in cases.GEMM_CASES
                               if c["dtype"] == "int8d" and "dtype_b" not in c],
                         ids=lambda c: c["key"])
def test_torch_port_matches_reference(golden, c):
    """The torch-CPU port that bench.py times as the CPU baseline gives the
    reference's packed result bit for bit (int8d, all configs[1]-style cases)."""
    from oracle import port_torch as PT
    a, b = cases.make_gemm_inputs(c)
    M, K, N = c["M"], c["K"], c["N"]
    ca, sa, _ = PT.quantize_int(a, 8, c["block"])
    cb, sb, _ = PT.quantize_int(b, 8, c["block"])
    codes, cs = PT.qscale_matmul(ca, sa, cb, sb, M, K, N, c["block"], 16)
    assert np.array_equal(PT.pack16(codes).numpy(), golden[f"{c['key']}/c_packed"])
    assert np.array_equal(cs.numpy().view(np.uint32), golden[f"{c['key']}/c_scales"].view(np.uint32))
