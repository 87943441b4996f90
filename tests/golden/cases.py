"""Seeded inputs shared by the golden generator and the tests.

Inputs come from torch's CPU generator, which is deterministic across
machines, so the fixtures store only the reference's outputs.
"""
import torch
import torch.nn as nn


def _randn(shape, seed, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(*shape, generator=g) * scale


def make_input(c):
    kind = c.get("dist", "normal")
    if kind == "config1":
        torch.manual_seed(0)
        return torch.randn(512, 512)
    if kind == "zeros":
        return torch.zeros(*c["shape"])
    if kind == "student_t":
        torch.manual_seed(c["seed"])
        x = torch.distributions.StudentT(3.0).sample(c["shape"])
    elif kind == "outlier":
        x = _randn(c["shape"], c["seed"], 0.02)
        g = torch.Generator().manual_seed(c["seed"] + 100)
        cols = torch.randperm(x.shape[-1], generator=g)[: max(1, x.shape[-1] // 64)]
        x[..., cols] *= 25.0
    else:
        x = _randn(c["shape"], c["seed"])
    if c.get("in_dtype") == "bf16":
        x = x.bfloat16()
    return x


def _q(key, dtype, block, **kw):
    d = {"key": key, "dtype": dtype, "block": block}
    d.update(kw)
    return d


QUANT_CASES = []
for _dt in ("int8d", "int4d", "int2d", "int1d", "float4d"):
    QUANT_CASES.append(_q(f"c1_{_dt}", _dt, 128, dist="config1"))
    for _blk in (32, 64, 256):
        QUANT_CASES.append(_q(f"b{_blk}_{_dt}", _dt, _blk, shape=(16, 512), seed=3 + _blk))
    QUANT_CASES.append(_q(f"ragged_{_dt}", _dt, 128, shape=(37, 53), seed=7))
    QUANT_CASES.append(_q(f"ragged64_{_dt}", _dt, 64, shape=(1001,), seed=8))
    QUANT_CASES.append(_q(f"tiny_{_dt}", _dt, 128, shape=(5,), seed=9))
    QUANT_CASES.append(_q(f"zeros_{_dt}", _dt, 128, shape=(4, 128), dist="zeros"))
    QUANT_CASES.append(_q(f"studt_{_dt}", _dt, 32, shape=(8192,), dist="student_t", seed=5))
    QUANT_CASES.append(_q(f"bf16_{_dt}", _dt, 128, shape=(16, 256), seed=10, in_dtype="bf16"))
    QUANT_CASES.append(_q(f"odd_block_{_dt}", _dt, 100, shape=(7, 90), seed=12))
# Hadamard variants
QUANT_CASES += [
    _q("h_int4dh_4x256", "int4dh", 128, shape=(4, 256), seed=20),
    _q("h_int4dh_16x1024", "int4dh", 128, shape=(16, 1024), seed=21, dist="outlier"),
    _q("h_int8dh_3x100", "int8dh", 64, shape=(3, 100), seed=22),
    _q("h_float4dh_2x512", "float4dh", 32, shape=(2, 512), seed=23),
    _q("h_int2dh_1d300", "int2dh", 64, shape=(300,), seed=24),
    _q("h_int1dh_8x128", "int1dh", 128, shape=(8, 128), seed=25),
    _q("h_int4dh_8x8192", "int4dh", 128, shape=(8, 8192), seed=26, dist="outlier"),
    _q("h_int8dh_bf16", "int8dh", 128, shape=(4, 512), seed=27, in_dtype="bf16"),
]


GEMM_CASES = [
    {"key": "g_c1_int8d", "dtype": "int8d", "block": 128, "dist": "config1", "M": 64, "K": 128, "N": 64},
    {"key": "g_int8d_128x256x128", "dtype": "int8d", "block": 128, "M": 128, "K": 256, "N": 128, "seed": 30},
    {"key": "g_int8d_256x512x256", "dtype": "int8d", "block": 128, "M": 256, "K": 512, "N": 256, "seed": 31},
    {"key": "g_int8d_b64", "dtype": "int8d", "block": 64, "M": 64, "K": 128, "N": 64, "seed": 32},
    {"key": "g_int4d_32x64x32", "dtype": "int4d", "block": 128, "M": 32, "K": 64, "N": 32, "seed": 33},
    {"key": "g_int4d_128x256x128", "dtype": "int4d", "block": 128, "M": 128, "K": 256, "N": 128, "seed": 34},
    {"key": "g_int2d_b64", "dtype": "int2d", "block": 64, "M": 64, "K": 128, "N": 64, "seed": 35},
    {"key": "g_int1d_b32", "dtype": "int1d", "block": 32, "M": 32, "K": 64, "N": 32, "seed": 36},
    {"key": "g_int8d_ragged", "dtype": "int8d", "block": 128, "M": 16, "K": 200, "N": 48, "seed": 37},
    # float-kind and variant operands: the reference multiplies their raw
    # sign-extended codes like int codes (mxtorch.py:5563-5573)
    {"key": "g_float4d_128x256x128", "dtype": "float4d", "block": 128, "M": 128, "K": 256, "N": 128, "seed": 38},
    {"key": "g_float4d_ragged", "dtype": "float4d", "block": 128, "M": 16, "K": 200, "N": 48, "seed": 39},
    {"key": "g_int4dh_128x256x128", "dtype": "int4dh", "block": 128, "M": 128, "K": 256, "N": 128, "seed": 46},
    {"key": "g_int4d_x_float4d", "dtype": "int4d", "dtype_b": "float4d", "block": 128, "M": 64, "K": 128, "N": 64, "seed": 47},
    {"key": "g_int2dh_b64", "dtype": "int2dh", "block": 64, "M": 64, "K": 128, "N": 64, "seed": 48},
]


def make_gemm_inputs(c):
    if c.get("dist") == "config1":
        torch.manual_seed(0)
        torch.randn(512, 512)
        return torch.randn(c["M"], c["K"]), torch.randn(c["K"], c["N"])
    g = torch.Generator().manual_seed(c["seed"])
    return (torch.randn(c["M"], c["K"], generator=g),
            torch.randn(c["K"], c["N"], generator=g))


LINEAR_CASES = [
    {"key": "l_int4d", "dtype": "int4d", "block": 128, "in": 256, "out": 384, "M": 5, "seed": 40},
    {"key": "l_int4d_bf16", "dtype": "int4d", "block": 128, "in": 256, "out": 384, "M": 3, "seed": 41, "x_dtype": "bf16"},
    {"key": "l_int8d", "dtype": "int8d", "block": 128, "in": 128, "out": 256, "M": 4, "seed": 42},
    {"key": "l_int2d", "dtype": "int2d", "block": 64, "in": 128, "out": 128, "M": 2, "seed": 43},
    {"key": "l_int1d", "dtype": "int1d", "block": 128, "in": 128, "out": 256, "M": 2, "seed": 44},
    {"key": "l_float4d", "dtype": "float4d", "block": 128, "in": 256, "out": 128, "M": 7, "seed": 45},
]


def make_linear_inputs(c):
    g = torch.Generator().manual_seed(c["seed"])
    lin = nn.Linear(c["in"], c["out"], bias=False)
    with torch.no_grad():
        lin.weight.copy_(torch.randn(c["out"], c["in"], generator=g) * 0.02)
    x = torch.randn(c["M"], c["in"], generator=g)
    if c.get("x_dtype") == "bf16":
        x = x.bfloat16()
    return lin, x


# cases whose full-size fp32 intermediates are not stored in the fixture
BIG_KEYS = {c["key"] for c in QUANT_CASES if c.get("dist") == "config1"} | {"h_int4dh_8x8192"}
