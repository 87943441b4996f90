"""mxb_linear_wonly_noalloc: the decode linear for callers that cannot
allocate device memory (pre-planned buffers, fixed pools, FFI hosts without
a CUDA allocator).  It must give the same result as mxb_linear_wonly, which
takes a caller-allocated workspace, within the linear tolerance of the other
tests: |y_a - y_b| <= 1e-5 * (|x| @ |W|) per element.  Two calls in a row
check that the shared internal scratch is reused correctly.

Collected last on purpose (file name), so a stop-at-first-failure run has
already run every other test."""
import pytest
import torch

import qtpytorch_b200 as mxb
from qtpytorch_b200 import _lib as L
from qtpytorch_b200 import ops

pytestmark = pytest.mark.gpu

LIN_TOL = 1e-5


def _noalloc(x, w, N, dt):
    K = x.shape[-1]
    M = x.numel() // K
    y = torch.empty(M, N, dtype=torch.float32, device=x.device)
    rc = L.load().mxb_linear_wonly_noalloc(
        L.ptr(x), L.BF16 if x.dtype == torch.bfloat16 else L.F32, M, K, L.ptr(w._mx_packed),
        L.ptr(w._mx_scales), N, dt.bits, L.KIND_FLOAT if dt.is_float else L.KIND_INT,
        w._mx_block, L.ptr(y), L.stream_of(x.device))
    L.check(rc, "mxb_linear_wonly_noalloc")
    return y


# The last case goes through the CUDA-core GEMV (float4 codes) whose own
# plan, 52 K splits of 80 rows, needs 36 MiB of partial sums: the entry point
# must lengthen the splits (to 256 rows, 11.3 MiB) to fit its 16 MiB array.
@pytest.mark.parametrize("M,K,N,dt", [(1, 4096, 11008, "int4d"), (16, 4096, 11008, "int4d"),
                                      (3, 512, 768, "int8d"), (5, 256, 384, "float4d"),
                                      (16, 4096, 11008, "float4d")])
def test_noalloc_matches_workspace_path(M, K, N, dt):
    d = mxb.get_mx_dtype(dt)
    g = torch.Generator().manual_seed(M + K)
    w = mxb.mx_tensor.quantize((torch.randn(K, N, generator=g) * 0.02).cuda(), d, 128)
    wdq = w.dequantize()
    for call in range(2):
        x = torch.randn(M, K, generator=g).bfloat16().cuda()
        ref = ops.linear_wonly(x, w._mx_packed, w._mx_scales, K, N, d, 128)
        y = _noalloc(x, w, N, d)
        torch.cuda.synchronize()
        bound = x.float().abs() @ wdq.abs()
        err = (y - ref).abs()
        assert torch.all(err <= LIN_TOL * bound + 1e-30), (call, float((err / bound).max()))
        # and against float64 x @ dequant(W^T) on sampled columns
        cols = torch.arange(0, N, max(1, N // 97), device=x.device)
        y64 = x.double() @ wdq[:, cols].double()
        err64 = (y[:, cols].double() - y64).abs()
        assert torch.all(err64 <= LIN_TOL * bound[:, cols].double() + 1e-30), call


def test_noalloc_rejects_partials_beyond_the_array():
    """float4d M=16, K=8192, N=32768: even 256-row K splits need 32 x 16 x
    32768 x 4 bytes = 64 MiB of partial sums, more than the 16 MiB array, so
    the call returns MXB_E_WORKSPACE (-7) before launching anything (the
    buffers are small stand-ins: nothing is read or written)."""
    w = torch.zeros(1 << 20, dtype=torch.int8, device="cuda")
    s = torch.ones(1 << 16, device="cuda")
    x = torch.zeros(16, 8192, dtype=torch.bfloat16, device="cuda")
    y = torch.empty(1 << 16, device="cuda")
    n0 = L.load().mxb_launch_count()
    rc = L.load().mxb_linear_wonly_noalloc(L.ptr(x), L.BF16, 16, 8192, L.ptr(w), L.ptr(s),
                                           32768, 4, L.KIND_FLOAT, 128, L.ptr(y),
                                           L.stream_of(x.device))
    assert rc == -7
    assert L.load().mxb_launch_count() == n0


def test_noalloc_rejects_non_gemv_shapes():
    w = mxb.mx_tensor.quantize(torch.randn(256, 384).cuda(), mxb.int4d, 128)
    x = torch.randn(32, 256).cuda()  # M > 16 is not a split-K GEMV shape
    y = torch.empty(32, 384, device="cuda")
    rc = L.load().mxb_linear_wonly_noalloc(L.ptr(x), L.F32, 32, 256, L.ptr(w._mx_packed),
                                           L.ptr(w._mx_scales), 384, 4, L.KIND_INT, 128,
                                           L.ptr(y), L.stream_of(x.device))
    assert rc == -1
