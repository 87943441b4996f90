"""tcgen05 weight-only GEMM (prefill regime) at the configs[2] size and the
decode GEMV beside it: parity mode within 1e-5 of |x| @ |W| per element
against an fp64 reference on sampled output columns; fast mode within the
bf16 rounding of the weights."""
import numpy as np
import pytest
import torch

import qtpytorch_b200 as mxb
from qtpytorch_b200 import _lib as L
from qtpytorch_b200 import ops

pytestmark = pytest.mark.gpu

LIN_TOL = 1e-5
FAST_TOL = 2.0 ** -8  # one bf16 rounding of each dequantized weight


@pytest.fixture(scope="module")
def llama_proj():
    # W ~ N(0, 0.02) [out=11008, in=4096], int4d block 128
    g = torch.Generator().manual_seed(1)
    w = torch.randn(11008, 4096, generator=g) * 0.02
    lin = torch.nn.Linear(4096, 11008, bias=False)
    with torch.no_grad():
        lin.weight.copy_(w)
    ml = mxb.mx_linear.from_linear(lin.cuda(), mxb.int4d, 128)
    wdq = ml._mx_weight.dequantize()  # [K, N] fp32, the reference's weight
    return ml, wdq


def _check_cols(y, x, wdq, tol, cols):
    x64 = x.float().cpu().numpy().astype(np.float64)
    w64 = wdq[:, cols].cpu().numpy().astype(np.float64)
    ref = x64 @ w64
    bound = np.abs(x64) @ np.abs(w64)
    err = np.abs(y[:, cols].cpu().numpy().astype(np.float64) - ref)
    worst = float((err / (bound + 1e-30)).max())
    assert np.all(err <= tol * bound + 1e-30), worst
    return worst


@pytest.mark.parametrize("M", [1, 16, 128, 2048])
def test_config3_parity(llama_proj, M):
    ml, wdq = llama_proj
    g = torch.Generator().manual_seed(2 + M)
    x = torch.randn(M, 4096, generator=g).bfloat16().cuda()
    y = ml(x)
    assert L.load().mxb_device_error(1) == 0
    cols = np.sort(np.random.default_rng(M).choice(11008, 96, replace=False))
    cols = np.concatenate([[0], cols, [11007]])
    _check_cols(y, x, wdq, LIN_TOL, cols)


def test_config3_fast_mode(llama_proj):
    ml, wdq = llama_proj
    x = torch.randn(512, 4096).bfloat16().cuda()
    y = ops.linear_wonly(x, ml._mx_weight._mx_packed, ml._mx_weight._mx_scales, 4096, 11008,
                         mxb.int4d, 128, mode=L.MODE_FAST)
    assert L.load().mxb_device_error(1) == 0
    cols = np.arange(0, 11008, 97)
    _check_cols(y, x, wdq, FAST_TOL, cols)


def test_prefill_matches_generic_kernel():
    """The tcgen05 path and the CUDA-core kernel agree to the parity bound
    (an fp32 x routes to the CUDA-core kernel)."""
    g = torch.Generator().manual_seed(5)
    w = mxb.mx_tensor.quantize((torch.randn(1024, 640, generator=g) * 0.02).cuda(), mxb.int8d, 128)
    x = torch.randn(300, 1024, generator=g).bfloat16().cuda()
    y_tc = ops.linear_wonly(x, w._mx_packed, w._mx_scales, 1024, 640, mxb.int8d, 128)
    y_cc = ops.linear_wonly(x.float(), w._mx_packed, w._mx_scales, 1024, 640, mxb.int8d, 128)
    bound = x.float().abs() @ w.dequantize().abs()
    assert torch.all((y_tc - y_cc).abs() <= 2 * LIN_TOL * bound + 1e-30)
