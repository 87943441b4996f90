"""tcgen05 packed GEMM: bit-exact against the oracle and the CUDA-core kernel,
at the golden sizes and at the full configs[1] size (4096^3)."""
import numpy as np
import pytest
import torch

import qtpytorch_b200 as mxb
from oracle import mx_oracle as O
from qtpytorch_b200 import _lib as L
from qtpytorch_b200 import ops

pytestmark = pytest.mark.gpu


def _u32(a):
    return np.ascontiguousarray(a).view(np.uint32)


def _device_ok():
    assert L.load().mxb_device_error(1) == 0


def _generic_c(qa, qb, M, K, N, bits):
    """fp32 C from the CUDA-core kernel (block != 128 forces it... so call with
    a scale count that is valid but through a misaligned copy)."""
    lib = L.load()
    # a 1-byte offset view of A makes the TMA path ineligible for int8
    dev = qa._mx_packed.device
    buf = torch.empty(qa._mx_packed.numel() + 16, dtype=torch.int8, device=dev)
    a_off = buf[1:1 + qa._mx_packed.numel()]
    a_off.copy_(qa._mx_packed)
    c = torch.empty(M, N, dtype=torch.float32, device=dev)
    wsb = lib.mxb_qgemm_workspace_size(M, K, N, bits, 128)
    ws = L.workspace(wsb, dev)
    rc = lib.mxb_qgemm(L.ptr(a_off), L.ptr(qa._mx_scales), qa._mx_scales.numel(),
                       L.ptr(qb._mx_packed), L.ptr(qb._mx_scales), qb._mx_scales.numel(),
                       M, K, N, bits, 128, 32, None, None, L.ptr(c), L.ptr(ws), wsb,
                       L.stream_of(dev))
    L.check(rc, "generic qgemm")
    return c


@pytest.mark.parametrize("M,K,N", [(128, 128, 128), (128, 256, 128), (256, 512, 384),
                                   (384, 1024, 256)])
@pytest.mark.parametrize("dt", ["int8d", "int4d", "int2d", "int1d"])
def test_tc_qgemm_matches_oracle(M, K, N, dt):
    d = mxb.get_mx_dtype(dt)
    g = torch.Generator().manual_seed(M * 7 + K + N)
    a = torch.randn(M, K, generator=g)
    b = torch.randn(K, N, generator=g)
    qa = mxb.mx_tensor.quantize(a.cuda(), d, 128)
    qb = mxb.mx_tensor.quantize(b.cuda(), d, 128)
    out_bits = mxb.optimal_output_dtype("matmul", d, d).bits
    cp, cs, c32 = ops.qgemm(qa._mx_packed, qa._mx_scales, qb._mx_packed, qb._mx_scales,
                            M, K, N, d.bits, 128, out_bits, want_f32=True)
    _device_ok()
    pa, sa, _ = O.quantize(a.numpy(), d.bits, "int", 128)
    pb, sb, _ = O.quantize(b.numpy(), d.bits, "int", 128)
    codes, cso, C = O.qscale_matmul(O.unpack(pa, d.bits, M * K), sa, O.unpack(pb, d.bits, K * N),
                                    sb, M, K, N, 128, out_bits)
    assert np.array_equal(_u32(c32.cpu().numpy()), _u32(C))
    assert np.array_equal(_u32(cs.cpu().numpy()), _u32(cso))
    assert np.array_equal(cp.cpu().numpy(), O.pack(codes, out_bits))


def test_tc_qgemm_full_size_4096():
    """bit-exact against the CUDA-core kernel over the whole C, and
    against the oracle on sampled rows (rows of C depend only on rows of A)."""
    M = N = K = 4096
    torch.manual_seed(0)
    a = torch.randn(M, K)
    b = torch.randn(K, N)
    qa = mxb.mx_tensor.quantize(a.cuda(), mxb.int8d, 128)
    qb = mxb.mx_tensor.quantize(b.cuda(), mxb.int8d, 128)
    cp, cs, c32 = ops.qgemm(qa._mx_packed, qa._mx_scales, qb._mx_packed, qb._mx_scales,
                            M, K, N, 8, 128, 16, want_f32=True)
    _device_ok()
    cg = _generic_c(qa, qb, M, K, N, 8)
    assert torch.equal(c32.view(torch.int32), cg.view(torch.int32))
    rows = np.sort(np.random.default_rng(0).choice(M, 48, replace=False))
    rows = np.concatenate([[0], rows, [M - 1]])
    pa = qa._mx_packed.cpu().numpy().reshape(M, K)[rows]
    sa = qa._mx_scales.cpu().numpy().reshape(M, K // 128)[rows]
    pb = qb._mx_packed.cpu().numpy()
    sb = qb._mx_scales.cpu().numpy()
    codes, cso, C = O.qscale_matmul(pa.astype(np.int32), sa.reshape(-1), pb.astype(np.int32), sb,
                                    len(rows), K, N, 128, 16)
    assert np.array_equal(_u32(c32.cpu().numpy()[rows]), _u32(C))
    # requantized int16 codes of those rows (each row = N/128 whole blocks)
    got = O.unpack(cp.cpu().numpy(), 16, M * N).reshape(M, N)[rows]
    assert np.array_equal(got.reshape(-1), codes)
    assert np.array_equal(_u32(cs.cpu().numpy().reshape(M, N // 128)[rows].reshape(-1)), _u32(cso))


def test_tc_qgemm_through_mx_tensor_matmul(golden):
    import cases
    c = [c for c in cases.GEMM_CASES if c["key"] == "g_int8d_256x512x256"][0]
    a, b = cases.make_gemm_inputs(c)
    qc = mxb.mx_tensor.quantize(a.cuda(), mxb.int8d) @ mxb.mx_tensor.quantize(b.cuda(), mxb.int8d)
    _device_ok()
    assert np.array_equal(qc._mx_packed.cpu().numpy(), golden[f"{c['key']}/c_packed"])
