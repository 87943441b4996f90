"""The C-ABI library loads, exports every declared symbol, and validates
arguments before touching the GPU (no compute calls here)."""
import ctypes
import os
import re

import pytest

from qtpytorch_b200 import _lib as L

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    names = set()
    for f in os.listdir(os.path.join(ROOT, "include")):
        if f.endswith(".h"):
            src = open(os.path.join(ROOT, "include", f)).read()
            names |= set(re.findall(r"^\s*(?:[\w\*\s]+?)\b(mxb_\w+)\s*\(", src, re.M))
    return names


def test_header_declares_entry_points():
    d = _declared()
    assert {"mxb_quantize", "mxb_dequantize", "mxb_qgemm", "mxb_linear_wonly"} <= d


def test_library_exports_every_declared_symbol():
    lib = L.load()
    for name in _declared():
        assert hasattr(lib, name), name
    assert set(L.PROTOTYPES) >= _declared() - {"mxb_set_cuda_error"}


def test_version_and_sizes():
    lib = L.load()
    assert lib.mxb_version() >= 100
    # nb*block codes, padded
    assert lib.mxb_packed_bytes(262144, 8, 128) == 262144
    assert lib.mxb_packed_bytes(1961, 4, 128) == 16 * 128 // 2
    assert lib.mxb_packed_bytes(5, 1, 128) == 16
    assert lib.mxb_packed_bytes(100 * 7, 1, 100) == 88  # ceil(700/8)
    assert lib.mxb_packed_bytes(4096, 16, 128) == 4096 * 2
    assert lib.mxb_packed_bytes(10, 3, 128) == 0
    assert lib.mxb_quantize_workspace_size(4096, 64, 4, 0, 0, 128) == 0
    assert lib.mxb_quantize_workspace_size(700, 90, 4, 0, 0, 100) == 7 * 4
    assert lib.mxb_linear_wonly_workspace_size(1, 4096, 11008, 4, 0, 128, 0) > 0


def test_argument_errors_need_no_gpu():
    lib = L.load()
    p = ctypes.c_void_p(16)
    # unsupported widths / kinds are rejected before any CUDA call
    assert lib.mxb_quantize(p, 0, 128, 128, 3, 0, 0, 128, None, p, p, None, 0, None) == -2
    assert lib.mxb_quantize(p, 0, 128, 128, 8, 1, 0, 128, None, p, p, None, 0, None) == -2
    assert lib.mxb_quantize(p, 0, 128, 128, 8, 0, 7, 128, None, p, p, None, 0, None) == -2
    assert lib.mxb_quantize(p, 0, 128, 128, 8, 0, 0, 0, None, p, p, None, 0, None) == -1
    assert lib.mxb_quantize(None, 0, 128, 128, 8, 0, 0, 128, None, p, p, None, 0, None) == -6
    assert lib.mxb_quantize(p, 0, 0, 1, 8, 0, 0, 128, None, p, p, None, 0, None) == 0
    assert lib.mxb_dequantize(p, p, 128, 128, 5, 0, 0, 128, None, p, None) == -2
    assert lib.mxb_qgemm(p, p, 1, p, p, 1, 64, 128, 64, 3, 128, 16, p, p, None, None, 0, None) == -2
    assert lib.mxb_qgemm(p, p, 1, p, p, 1, 64, 128, 64, 8, 128, 16, p, p, None, None, 0, None) == -7
    assert lib.mxb_linear_wonly(p, 0, 4, 128, p, p, 64, 4, 0, 128, 9, p, None, 0, None) == -6
    assert lib.mxb_linear_wonly(p, 0, 4, 128, p, p, 128, 4, 0, 128, 0, p, None, 0, None) == -7
    assert lib.mxb_hadamard_rows(p, 1, 1 << 16, p, 0, p, None) == -1


def test_dynamic_and_epilogue_argument_errors_need_no_gpu():
    lib = L.load()
    p = ctypes.c_void_p(16)
    # dynamic quantize: int1 (max_int 0 in the reference) and odd widths rejected
    assert lib.mxb_dynamic_quantize(p, 0, 128, 128, 1, p, p, None, 0, None) == -2
    assert lib.mxb_dynamic_quantize(p, 0, 128, 128, 3, p, p, None, 0, None) == -2
    assert lib.mxb_dynamic_quantize(p, 0, 128, 0, 8, p, p, None, 0, None) == -1
    assert lib.mxb_dynamic_quantize(p, 0, 128, 1 << 31, 8, p, p, None, 0, None) == -1
    assert lib.mxb_dynamic_quantize(p, 9, 128, 128, 8, p, p, None, 0, None) == -2
    assert lib.mxb_dynamic_quantize(None, 0, 128, 128, 8, p, p, None, 0, None) == -6
    assert lib.mxb_dynamic_quantize(p, 0, 0, 128, 8, p, p, None, 0, None) == 0
    assert lib.mxb_dynamic_quantize_workspace_size(1 << 20, 128) == 0
    assert lib.mxb_dynamic_quantize_workspace_size(4096 * 3, 4096) == 3 * 4
    # fused epilogues
    assert lib.mxb_dequantize_relu(p, p, 128, 3, 0, 128, p, None) == -2
    assert lib.mxb_dequantize_relu(p, p, -1, 8, 0, 128, p, None) == -1
    assert lib.mxb_dequantize_relu(p, None, 128, 8, 0, 128, p, None) == -6
    assert lib.mxb_dequantize_silu_mul(p, p, p, p, 128, 8, 1, 128, p, None) == -2
    assert lib.mxb_dequantize_silu_mul(p, p, None, p, 128, 8, 0, 128, p, None) == -6
    assert lib.mxb_dequantize_silu_mul(p, p, p, p, 0, 8, 0, 128, p, None) == 0
