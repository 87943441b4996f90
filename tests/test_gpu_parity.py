"""CUDA path vs the reference's outputs (golden fixtures) and the oracle.

Bit-exact: packed codes, scales, dequantized values, the matmul's int32
K-block partials, fp32 accumulator and requantized codes.  Weight-only
linear (fp32 output): |y - y64| <= 1e-5 * (|x| @ |W|) per element.
"""
import numpy as np
import pytest
import torch

import cases
import qtpytorch_b200 as mxb
from oracle import mx_oracle as O
from qtpytorch_b200 import _lib as L
from qtpytorch_b200 import ops
from qtpytorch_b200.dtypes import get_mx_dtype

pytestmark = pytest.mark.gpu

LIN_TOL = 1e-5  # per element, relative to |x| @ |W_dq|


def _u32(a):
    return np.ascontiguousarray(a).view(np.uint32)


@pytest.mark.parametrize("c", cases.QUANT_CASES, ids=lambda c: c["key"])
def test_quantize_bit_exact(golden, c):
    dt = get_mx_dtype(c["dtype"])
    x = cases.make_input(c).cuda()
    q = mxb.mx_tensor.quantize(x, dt, c["block"])
    k = c["key"]
    assert q._mx_n == int(golden[f"{k}/n"])
    assert np.array_equal(_u32(q._mx_scales.cpu().numpy()), _u32(golden[f"{k}/scales"]))
    assert np.array_equal(q._mx_packed.cpu().numpy(), golden[f"{k}/packed"])
    dq = q.dequantize()
    assert dq.shape == x.shape
    if f"{k}/dequant" in golden:
        assert np.array_equal(_u32(dq.cpu().numpy()), _u32(golden[f"{k}/dequant"]))
    else:
        signs = None
        if dt.is_hadamard:
            signs = mxb.sign_vector(ops.row_len_of(x.shape), dt.hadamard_seed).numpy()
        ref = O.dequantize(golden[f"{k}/packed"], golden[f"{k}/scales"], dt.bits, dt.kind,
                           tuple(x.shape), c["block"], dt.is_hadamard, signs)
        assert np.array_equal(_u32(dq.cpu().numpy()), _u32(ref))


@pytest.mark.parametrize("n", [8, 1000, 1024, 1032, 4104, 33000, (1 << 20) + 24])
@pytest.mark.parametrize("dt", ["int1d", "int2d", "int4d", "int8d", "float4d"])
@pytest.mark.parametrize("block", [8, 32, 128])
@pytest.mark.parametrize("in_dt", [torch.float32, torch.bfloat16])
def test_dequantize_ragged(n, dt, block, in_dt):
    """Vectorised quantize and dequantize kernels at lengths that end inside
    a 1024-element chunk, a packed word and a scale block."""
    d = get_mx_dtype(dt)
    g = torch.Generator().manual_seed(n + block)
    x = torch.randn(n, generator=g).to(in_dt)
    q = mxb.mx_tensor.quantize(x.cuda(), d, block)
    p, s, _ = O.quantize(x.float().numpy(), d.bits, d.kind, block)
    assert np.array_equal(q._mx_packed.cpu().numpy(), p)
    assert np.array_equal(_u32(q._mx_scales.cpu().numpy()), _u32(s))
    dq = q.dequantize().cpu().numpy()
    ref = O.dequantize(q._mx_packed.cpu().numpy(), q._mx_scales.cpu().numpy(), d.bits, d.kind,
                       (n,), block)
    assert np.array_equal(_u32(dq), _u32(ref))


@pytest.mark.parametrize("in_dt", [torch.float32, torch.bfloat16])
def test_quantize_float4_near_boundaries(in_dt):
    """float4 codes for values within 4 ulp of every rounding boundary (and
    of a 2^-20 quotient) times the block absmax, over divisors with extreme
    mantissas (all ones, all zeros) and exponents 2^-39..2^127, plus signed
    zeros and a subnormal: the bucket of the IEEE quotient everywhere."""
    rng = np.random.default_rng(11)
    nblk, block = 8192, 128
    mant = rng.integers(0, 1 << 23, nblk, dtype=np.uint32)
    mant[:512] = 0x7FFFFF
    mant[512:1024] = 0
    mant[1024:1536] = 0x7FFFFF ^ rng.integers(0, 8, 512, dtype=np.uint32)
    ex = rng.integers(127 - 39, 127 + 127, nblk, dtype=np.uint32)
    ex[:64] = 127 + 125
    ex[64:128] = 127 + 126
    a = ((ex << 23) | mant).view(np.float32)
    if in_dt == torch.bfloat16:
        a = (a.view(np.uint32) & 0xFFFF0000).view(np.float32)
    mids = O.minifloat4_mids()
    targets = np.concatenate([mids[mids > 0], np.float32([2.0 ** -20])]).astype(np.float32)
    prod = (a[:, None].astype(np.float64) * targets[None, :]).astype(np.float32)
    offs = np.arange(-4, 5, dtype=np.int64)
    bits = prod.view(np.int32)[:, :, None].astype(np.int64) + offs[None, None, :]
    vals = bits.astype(np.int32).view(np.float32).reshape(nblk, -1)
    vals = np.abs(vals) * np.where(rng.random(vals.shape) < 0.5, -1, 1).astype(np.float32)
    blk = np.zeros((nblk, block), np.float32)
    take = min(vals.shape[1], block - 4)
    blk[:, 0] = a * np.where(rng.random(nblk) < 0.5, -1, 1).astype(np.float32)
    blk[:, 1:1 + take] = vals[:, :take]
    blk[:, block - 3] = 0.0
    blk[:, block - 2] = -0.0
    blk[:, block - 1] = np.float32(1e-45)
    x = torch.from_numpy(blk.reshape(-1)).to(in_dt)
    xf = x.float().numpy()
    assert np.all(np.abs(xf.reshape(nblk, block)).max(axis=1) == np.abs(xf.reshape(nblk, block)[:, 0]))
    d = get_mx_dtype("float4d")
    q = mxb.mx_tensor.quantize(x.cuda(), d, block)
    p, s, _ = O.quantize(xf, d.bits, d.kind, block)
    assert np.array_equal(q._mx_scales.cpu().numpy(), s)
    assert np.array_equal(q._mx_packed.cpu().numpy(), p)


@pytest.mark.parametrize("offset", [1, 3])
def test_quantize_unaligned_views(offset):
    # pointers not 16-byte aligned take the scalar-load path
    base = torch.randn(4 * 256 + offset, device="cuda")
    x = base[offset:]
    for dt in ("int8d", "int4d", "float4d"):
        d = get_mx_dtype(dt)
        q = mxb.mx_tensor.quantize(x, d, 128)
        p, s, _ = O.quantize(x.cpu().numpy(), d.bits, d.kind, 128)
        assert np.array_equal(q._mx_packed.cpu().numpy(), p)
        assert np.array_equal(q._mx_scales.cpu().numpy(), s)


def test_quantize_specials():
    x = torch.randn(8, 128)
    x[0, 3] = float("inf")
    x[1, :] = 0.0
    x[2, 5] = -0.0
    x[3, :] = 1e-30
    for dt in ("int8d", "int4d", "int2d", "int1d", "float4d"):
        d = get_mx_dtype(dt)
        q = mxb.mx_tensor.quantize(x.cuda(), d, 128)
        p, s, _ = O.quantize(x.numpy(), d.bits, d.kind, 128)
        assert np.array_equal(q._mx_packed.cpu().numpy(), p), dt
        assert np.array_equal(_u32(q._mx_scales.cpu().numpy()), _u32(s)), dt


def _float4_edge_input():
    """Rows of 128 whose quotients x / amax land exactly on, and one ulp either
    side of, each float4 bucket boundary (both signs), plus +-0, denormals,
    quotients that underflow to zero, and blocks holding inf / NaN."""
    # the fp32 midpoints of adjacent grid values, as the kernels compare them
    grid = np.array([0, 1, 2, 3, 4, 6, 8, 12], dtype=np.float32) / np.float32(12)
    mids = ((grid[:-1] + grid[1:]) * np.float32(0.5)).astype(np.float32)
    up = np.nextafter(mids, np.float32(np.inf))
    dn = np.nextafter(mids, np.float32(0))
    vals = np.concatenate([mids, up, dn]).astype(np.float32)
    vals = np.concatenate([vals, -vals, np.float32([0.0, -0.0, 1e-45, -1e-45, 1e-38, -1e-38])])
    rows = []
    for amax in (1.0, 3.0, 0.7, 1e-20, 2.0 ** 100):
        r = np.zeros(128, dtype=np.float32)
        r[0] = amax
        v = (vals.astype(np.float64) * amax).astype(np.float32)
        r[1:1 + len(v)] = v
        rows.append(r)
    r = np.zeros(128, dtype=np.float32)
    r[0] = 2.0 ** 100
    r[1:8] = [1e-45, -1e-45, 3e-45, 1e-40, -1e-40, 1e-38, 0.0]
    rows.append(r)
    r = np.linspace(-2, 2, 128).astype(np.float32)
    r[7] = np.inf
    r[9] = -np.inf
    rows.append(r)
    r = np.linspace(-2, 2, 128).astype(np.float32)
    r[4] = np.nan
    rows.append(r)
    return np.stack(rows)


@pytest.mark.parametrize("block", [32, 128])
def test_float4_bucket_table_cells(block):
    """Blocks with absmax 1 (so the quotient is the value itself): every
    float within 256 ulp of each 1/16-binade cell edge of the bucket table
    (2^-6 .. 4) and of each boundary, both signs, plus the zeros: codes
    equal the oracle's bucketize of the IEEE quotient."""
    edges = np.arange(0x7A0 - 16, 0x7F0 + 16, dtype=np.int64) << 19
    bnd = np.abs(O.minifloat4_mids()).view(np.int32).astype(np.int64)
    centres = np.unique(np.concatenate([edges, bnd]))
    bits = (centres[:, None] + np.arange(-256, 257, dtype=np.int64)[None, :]).reshape(-1)
    bits = bits[(bits >= 0) & (bits <= 0x3F800000)]
    v = bits.astype(np.int32).view(np.float32)
    v = np.concatenate([v, -v, np.float32([0.0, -0.0])])
    per = block - 1
    nb = -(-v.size // per)
    v = np.concatenate([v, np.zeros(nb * per - v.size, np.float32)]).reshape(nb, per)
    x = np.concatenate([np.ones((nb, 1), np.float32), v], axis=1).reshape(-1)
    d = get_mx_dtype("float4d")
    q = mxb.mx_tensor.quantize(torch.from_numpy(x).cuda(), d, block)
    p, s, _ = O.quantize(x, d.bits, d.kind, block)
    assert np.array_equal(q._mx_packed.cpu().numpy(), p)
    assert np.array_equal(_u32(q._mx_scales.cpu().numpy()), _u32(s))


def test_float4_bucket_boundaries():
    x = _float4_edge_input()
    d = get_mx_dtype("float4d")
    q = mxb.mx_tensor.quantize(torch.from_numpy(x).cuda(), d, 128)
    p, s, _ = O.quantize(x, d.bits, d.kind, 128)
    assert np.array_equal(q._mx_packed.cpu().numpy(), p)
    # bit-exact scales; a NaN block's scale is NaN (its payload is not compared)
    gs = q._mx_scales.cpu().numpy()
    nan = np.isnan(s)
    assert np.array_equal(np.isnan(gs), nan)
    assert np.array_equal(_u32(gs[~nan]), _u32(s[~nan]))


@pytest.mark.parametrize("c", [c for c in cases.QUANT_CASES if "h_" in c["key"]],
                         ids=lambda c: c["key"])
def test_hadamard_rotation_matches_reference(golden, c):
    dt = get_mx_dtype(c["dtype"])
    x = cases.make_input(c).float()
    k = c["key"]
    if f"{k}/rotated" not in golden:
        pytest.skip("rotation not stored for this size")
    xr = x if x.dim() >= 2 else x.reshape(1, -1)
    y = ops.hadamard_rows(xr.cuda(), dt.hadamard_seed, inverse=False)
    assert np.array_equal(_u32(y.cpu().numpy()), _u32(golden[f"{k}/rotated"]))


def test_hadamard_roundtrip_8192():
    # config-4 row length: unrotate(rotate(x)) == x to fp32 rounding
    x = torch.randn(16, 8192, device="cuda")
    y = ops.hadamard_rows(x, 1214670534, inverse=False)
    z = ops.hadamard_rows(y, 1214670534, inverse=True)
    assert torch.allclose(z, x, atol=1e-5, rtol=1e-5)
    r = O.rotate(x.cpu().numpy(), mxb.sign_vector(8192, 1214670534).numpy())
    assert np.array_equal(_u32(y.cpu().numpy()), _u32(r))


@pytest.mark.parametrize("c", cases.GEMM_CASES, ids=lambda c: c["key"])
def test_qgemm_bit_exact(golden, c):
    dt = get_mx_dtype(c["dtype"])
    a, b = cases.make_gemm_inputs(c)
    qa = mxb.mx_tensor.quantize(a.cuda(), dt, c["block"])
    qb = mxb.mx_tensor.quantize(b.cuda(), get_mx_dtype(c.get("dtype_b", c["dtype"])), c["block"])
    n0 = L.load().mxb_launch_count()
    qc = qa @ qb
    assert L.load().mxb_launch_count() > n0  # the library's kernels, no torch matmul
    k = c["key"]
    assert qc._mx_dtype.name == str(golden[f"{k}/c_dtype"])
    assert qc._mx_dtype.bits == int(golden[f"{k}/c_bits"])
    assert qc._mx_block == int(golden[f"{k}/c_block"])
    assert np.array_equal(_u32(qc._mx_scales.cpu().numpy()), _u32(golden[f"{k}/c_scales"]))
    assert np.array_equal(qc._mx_packed.cpu().numpy(), golden[f"{k}/c_packed"])
    if qc._mx_dtype.is_int:  # float8d results dequantize through the reference's fp8 grid
        assert np.array_equal(_u32(qc.dequantize().cpu().numpy()), _u32(golden[f"{k}/c_dequant"]))


def _linear_check(y, x, wdq, tol=LIN_TOL):
    y64, bound = O.linear_ref64(x, wdq)
    err = np.abs(y.astype(np.float64) - y64)
    assert np.all(err <= tol * bound + 1e-30), float((err / (bound + 1e-30)).max())
    return float((err / (bound + 1e-30)).max())


@pytest.mark.parametrize("c", cases.LINEAR_CASES, ids=lambda c: c["key"])
def test_mx_linear_matches_reference(golden, c):
    lin, x = cases.make_linear_inputs(c)
    dt = get_mx_dtype(c["dtype"])
    ml = mxb.mx_linear.from_linear(lin.cuda(), dt, c["block"])
    assert np.array_equal(ml._mx_weight._mx_packed.cpu().numpy(), golden[f"{c['key']}/w_packed"])
    y = ml(x.cuda())
    assert y.dtype == torch.float32 and y.shape == (c["M"], c["out"])
    wdq = O.dequantize(golden[f"{c['key']}/w_packed"], golden[f"{c['key']}/w_scales"], dt.bits,
                       dt.kind, (c["in"], c["out"]), c["block"])
    _linear_check(y.cpu().numpy(), x.float().numpy(), wdq)
    # the reference's own fp32 output agrees to the same tolerance
    yr = golden[f"{c['key']}/y"]
    y64, bound = O.linear_ref64(x.float().numpy(), wdq)
    assert np.all(np.abs(yr - y64) <= LIN_TOL * bound + 1e-30)


@pytest.mark.parametrize("M", [1, 3, 16, 17, 32, 64, 128])
@pytest.mark.parametrize("dt", ["int4d", "int8d", "int2d", "int1d", "float4d"])
def test_linear_shapes(M, dt):
    d = get_mx_dtype(dt)
    g = torch.Generator().manual_seed(M)
    w = torch.randn(384, 256, generator=g) * 0.02   # out=384, in=256
    x = torch.randn(M, 256, generator=g).bfloat16()
    lin = torch.nn.Linear(256, 384, bias=False)
    with torch.no_grad():
        lin.weight.copy_(w)
    ml = mxb.mx_linear.from_linear(lin.cuda(), d, 128)
    y = ml(x.cuda()).cpu().numpy()
    pw, sw, _ = O.quantize(w.t().contiguous().numpy(), d.bits, d.kind, 128)
    wdq = O.dequantize(pw, sw, d.bits, d.kind, (256, 384), 128)
    _linear_check(y, x.float().numpy(), wdq)


@pytest.mark.parametrize("M", [3, 5, 24, 32])
@pytest.mark.parametrize("dt", ["int4d", "int8d", "int2d", "int1d"])
def test_decode_tc_uneven_k(M, dt):
    """Decode shapes on the tcgen05 split-K kernel with a K (17 steps of 64)
    that does not divide evenly into the K chunks, block 256."""
    d = get_mx_dtype(dt)
    g = torch.Generator().manual_seed(100 + M)
    K, N = 1088, 640
    w = torch.randn(N, K, generator=g) * 0.02
    x = torch.randn(M, K, generator=g).bfloat16()
    lin = torch.nn.Linear(K, N, bias=False)
    with torch.no_grad():
        lin.weight.copy_(w)
    ml = mxb.mx_linear.from_linear(lin.cuda(), d, 256)
    y = ml(x.cuda()).cpu().numpy()
    assert L.load().mxb_device_error(1) == 0
    pw, sw, _ = O.quantize(w.t().contiguous().numpy(), d.bits, d.kind, 256)
    wdq = O.dequantize(pw, sw, d.bits, d.kind, (K, N), 256)
    _linear_check(y, x.float().numpy(), wdq)


@pytest.mark.parametrize("dt", ["int4d", "int4dh"])
def test_sharded_linear_single_rank_equals_module(dt):
    """The column-sharded linear at world 1 runs the same kernel (and the
    row unrotation for h dtypes) as mx_linear.forward."""
    from qtpytorch_b200 import parallel as P
    d = get_mx_dtype(dt)
    g = torch.Generator().manual_seed(9)
    lin = torch.nn.Linear(512, 640, bias=False)
    with torch.no_grad():
        lin.weight.copy_(torch.randn(640, 512, generator=g) * 0.02)
    ml = mxb.mx_linear.from_linear(lin.cuda(), d, 128)
    x = torch.randn(24, 512, generator=g).bfloat16().cuda()
    sw = P.ShardedLinearWeight.from_module(ml, 1, 0)
    y = P.sharded_linear(x, sw)
    assert torch.equal(y, ml(x))
    yb = P.sharded_linear(x, sw, out_dtype=torch.bfloat16)
    assert yb.dtype == torch.bfloat16 and torch.equal(yb, ml(x).bfloat16())


@pytest.mark.parametrize("M,K,N", [(256, 384, 256), (40, 256, 96)])  # tcgen05 / CUDA-core
@pytest.mark.parametrize("dt", ["int8d", "int4d", "int2d", "int1d"])
def test_qgemm_kmajor(M, K, N, dt):
    """k-major mode: B quantized along K (as B.t()).  Bit-exact against the
    oracle's K-block formula fed B^T's codes and scales transposed into the
    [K, N] / [K/block, N] layout, and within fp32 rounding of the fp64
    dequant(A) @ dequant(B)."""
    d = get_mx_dtype(dt)
    g = torch.Generator().manual_seed(M + N + d.bits)
    a = torch.randn(M, K, generator=g)
    b = torch.randn(K, N, generator=g)
    qa = mxb.mx_tensor.quantize(a.cuda(), d, 128)
    qbt = mxb.mx_tensor.quantize(b.t().contiguous().cuda(), d, 128)
    c = mxb.mx_matmul_kmajor(qa, qbt)
    ob = c._mx_dtype.bits  # a.bits + b.bits snapped (int16d for int8 x int8)
    c_packed, c_scales, c32 = ops.qgemm(qa._mx_packed, qa._mx_scales, qbt._mx_packed,
                                        qbt._mx_scales, M, K, N, d.bits, 128, ob,
                                        want_f32=True, b_kmajor=True)
    assert L.load().mxb_device_error(1) == 0
    kbn = K // 128
    a_codes = O.unpack(qa._mx_packed.cpu().numpy(), d.bits, M * K)
    bt_codes = O.unpack(qbt._mx_packed.cpu().numpy(), d.bits, N * K).reshape(N, K)
    if d.bits == 1:  # k-major mode counts 1-bit codes as +-1 (their dequantized meaning)
        a_codes = np.where(a_codes == 0, 1, -1).astype(a_codes.dtype)
        bt_codes = np.where(bt_codes == 0, 1, -1).astype(bt_codes.dtype)
    sbt = qbt._mx_scales.cpu().numpy().reshape(N, kbn)
    codes, cs, C = O.qscale_matmul(a_codes, qa._mx_scales.cpu().numpy(),
                                   np.ascontiguousarray(bt_codes.T).reshape(-1),
                                   np.ascontiguousarray(sbt.T).reshape(-1), M, K, N, 128, ob)
    assert np.array_equal(_u32(c32.cpu().numpy()), _u32(C))
    want = O.pack(codes, ob)
    assert np.array_equal(c_packed.cpu().numpy().view(want.dtype), want)
    assert np.array_equal(_u32(c_scales.cpu().numpy()), _u32(cs))
    assert np.array_equal(c._mx_packed.cpu().numpy(), c_packed.cpu().numpy())
    # every element met its own scale: the fp64 quantized product
    adq = O.dequant_flat(qa._mx_packed.cpu().numpy(), qa._mx_scales.cpu().numpy(), d.bits,
                         d.kind, M * K, 128).reshape(M, K).astype(np.float64)
    bdq = O.dequant_flat(qbt._mx_packed.cpu().numpy(), sbt.reshape(-1), d.bits, d.kind,
                         N * K, 128).reshape(N, K).astype(np.float64).T
    ref = adq @ bdq
    bound = np.abs(adq) @ np.abs(bdq)
    assert np.all(np.abs(C.astype(np.float64) - ref) <= 1e-5 * bound + 1e-30)


def test_qgemm_kmajor_rejects_straddling_blocks():
    qa = mxb.mx_tensor.quantize(torch.randn(8, 200).cuda(), mxb.int8d, 128)
    qbt = mxb.mx_tensor.quantize(torch.randn(16, 200).cuda(), mxb.int8d, 128)
    with pytest.raises(L.MxbError):
        mxb.mx_matmul_kmajor(qa, qbt)


@pytest.mark.parametrize("M", [1, 2])
@pytest.mark.parametrize("dt", ["int4d", "int8d"])
@pytest.mark.parametrize("K,N,block,x_dt", [
    (4096, 11008, 128, torch.bfloat16),   # configs[2]: 43 groups of 256 columns
    (1000, 640, 64, torch.float32),       # K not a multiple of 32, last group half wide
    (328, 512, 256, torch.bfloat16),      # group wider than N
    (96, 256, 32, torch.float32),         # fewer units than SMs
    (8192, 3072, 1024, torch.bfloat16),   # one scale per group row
])
def test_decode_gemv_shapes(M, dt, K, N, block, x_dt):
    """The decode GEMV (M <= 2, int4 / int8) at the configs[2] shape, ragged
    K, a 640-wide N, small K, blocks from 32 to 1024, fp32 and bf16 x; and a
    second call that reuses the workspace."""
    d = get_mx_dtype(dt)
    g = torch.Generator().manual_seed(K + N + M)
    w = torch.randn(K, N, generator=g) * 0.02
    q = mxb.mx_tensor.quantize(w.cuda(), d, block)
    wdq = O.dequantize(q._mx_packed.cpu().numpy(), q._mx_scales.cpu().numpy(), d.bits, d.kind,
                       (K, N), block)
    for call in range(2):
        x = torch.randn(M, K, generator=g).to(x_dt)
        y = ops.linear_wonly(x.cuda(), q._mx_packed, q._mx_scales, K, N, d, block)
        assert L.load().mxb_device_error(1) == 0
        _linear_check(y.cpu().numpy(), x.float().numpy(), wdq)


@pytest.mark.parametrize("d,rows", [(4096, 700), (8192, 600), (8192, 1777)])
def test_pipelined_wht_rows_bit_exact(d, rows):
    """Enough whole power-of-two rows for the pipelined row kernel (each
    persistent CTA copies its next row into shared memory while it
    transforms the current one), row counts that leave CTAs with different
    numbers of rows: rotation and unrotation bit-identical to the oracle,
    and no device error recorded."""
    seed = get_mx_dtype("int4dh").hadamard_seed
    g = torch.Generator().manual_seed(rows)
    x = torch.randn(rows, d, generator=g)
    signs = mxb.sign_vector(d, seed).numpy()
    L.load().mxb_device_error(1)
    rot = ops.hadamard_rows(x.cuda(), seed, inverse=False).cpu().numpy()
    assert np.array_equal(_u32(rot), _u32(O.rotate(x.numpy(), signs)))
    un = ops.hadamard_rows(x.cuda(), seed, inverse=True).cpu().numpy()
    assert np.array_equal(_u32(un), _u32(O.unrotate(x.numpy(), signs)))
    assert L.load().mxb_device_error(1) == 0


@pytest.mark.parametrize("dtn,block", [("int4dh", 128), ("int2dh", 32), ("float4dh", 128),
                                       ("int8dh", 64), ("int1dh", 128)])
def test_h_quantize_many_rows_bit_exact(dtn, block):
    """fp32 h quantize of 640 rows of 8192 with an outlier channel (the
    register-WHT kernel over many CTAs): packed codes and scales
    bit-identical to the oracle."""
    dt = get_mx_dtype(dtn)
    g = torch.Generator().manual_seed(block)
    x = torch.randn(640, 8192, generator=g)
    x[:, 17] *= 25.0  # an outlier channel
    signs = mxb.sign_vector(8192, dt.hadamard_seed).numpy()
    L.load().mxb_device_error(1)
    q = mxb.mx_tensor.quantize(x.cuda(), dt, block)
    p, s, _ = O.quantize(x.numpy(), dt.bits, dt.kind, block, True, signs)
    assert np.array_equal(q._mx_packed.cpu().numpy(), p)
    assert np.array_equal(_u32(q._mx_scales.cpu().numpy()), _u32(s))
    assert L.load().mxb_device_error(1) == 0


@pytest.mark.parametrize("d,dtn", [(2048, "int4dh"), (3000, "int4dh"), (4096, "int4dh"),
                                   (8192, "int4dh"), (12000, "int4dh"), (16384, "int4dh"),
                                   (4096, "int8dh"), (8192, "int8dh"), (8192, "int2dh"),
                                   (4096, "float4dh"), (16384, "int1dh")])
def test_register_wht_rows_bit_exact(d, dtn):
    """Row lengths whose transform runs in registers (padded lengths 2048 ..
    16384), rows loaded element-wise or in runs: rotation, unrotation, h
    quantize and h dequantize bit-identical to the oracle's stage order
    (mxtorch.py:2811-2904, 1720-1736)."""
    dt = get_mx_dtype(dtn)
    g = torch.Generator().manual_seed(d)
    x = torch.randn(6, d, generator=g)
    if dtn == "int8dh":  # bf16 rows through the quantizer's run loads
        x = x.bfloat16().float()
    signs = mxb.sign_vector(d, dt.hadamard_seed).numpy()
    rot = ops.hadamard_rows(x.cuda(), dt.hadamard_seed, inverse=False).cpu().numpy()
    assert np.array_equal(_u32(rot), _u32(O.rotate(x.numpy(), signs)))
    un = ops.hadamard_rows(x.cuda(), dt.hadamard_seed, inverse=True).cpu().numpy()
    assert np.array_equal(_u32(un), _u32(O.unrotate(x.numpy(), signs)))
    block = 128 if d % 128 == 0 else 8 if d % 8 == 0 else 100
    xq = x.bfloat16() if dtn == "int8dh" else x  # exact: x holds bf16 values there
    q = mxb.mx_tensor.quantize(xq.cuda(), dt, block)
    p, s, _ = O.quantize(x.numpy(), dt.bits, dt.kind, block, True, signs)
    assert np.array_equal(q._mx_packed.cpu().numpy(), p)
    assert np.array_equal(_u32(q._mx_scales.cpu().numpy()), _u32(s))
    ref = O.dequantize(p, s, dt.bits, dt.kind, (6, d), block, True, signs)
    assert np.array_equal(_u32(q.dequantize().cpu().numpy()), _u32(ref))
