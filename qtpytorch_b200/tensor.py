"""``mx_tensor``: a torch.Tensor subclass holding bit-packed codes + block scales.

Mirrors the reference's storage contract and API (mxtorch.py:6028-6425):
attributes ``_mx_packed`` (int8 bytes; int32 words for 16-bit codes),
``_mx_scales`` (fp32 [ceil(n/block)]), ``_mx_dtype``, ``_mx_orig_shape``,
``_mx_n``, ``_mx_block``; ``quantize`` / ``dequantize`` / ``@`` /
``__tensor_flatten__`` / ``__tensor_unflatten__``.  The arithmetic runs in
the mxb CUDA library.

Deliberate differences from the reference, all on purpose:
* reading tensor properties (``.device``, ``.requires_grad``) answers from
  the wrapper and does not dequantize (the reference dequantizes the whole
  tensor per read, mxtorch.py:6162-6165); ``requires_grad`` reads False, the
  value the reference ends up with, so ``A @ B`` takes the packed GEMM;
* ``dequantize`` of an ``h`` tensor with >= 2 dims inverts the rotation along
  the last dim, the one quantize rotated (the reference inverts along the
  flattened tensor, mxtorch.py:1583-1595, which does not invert it).
"""
from __future__ import annotations

import os
import re
from dataclasses import dataclass
from typing import Callable, List, Optional

import torch
from torch.utils._pytree import tree_map

from . import ops
from .dtypes import get_mx_dtype, mx_dtype, optimal_output_dtype

_STRICT = os.environ.get("MX_STRICT", "0") == "1"


class mx_tensor(torch.Tensor):
    """A quantized tensor that is a torch.Tensor (mxtorch.py:6028)."""

    def __new__(cls, packed: torch.Tensor, scales: torch.Tensor, mx_dtype: mx_dtype,
                orig_shape, n: int, block: int = 128, requires_grad: bool = False):
        dummy = torch.empty((), dtype=torch.float32, device=packed.device)
        inst = torch.Tensor._make_subclass(cls, dummy, False)
        inst._mx_packed = packed
        inst._mx_scales = scales
        inst._mx_dtype = get_mx_dtype(mx_dtype)
        inst._mx_orig_shape = torch.Size(orig_shape)
        inst._mx_n = int(n)
        inst._mx_block = int(block)
        return inst

    def __init__(self, *args, **kwargs):
        pass

    # ── tensor-subclass protocol (mxtorch.py:6058-6085) ──────────────────────
    def __tensor_flatten__(self):
        return ["_mx_packed", "_mx_scales"], {
            "mx_dtype": self._mx_dtype,
            "orig_shape": self._mx_orig_shape,
            "n": self._mx_n,
            "block": self._mx_block,
        }

    @staticmethod
    def __tensor_unflatten__(inner_tensors, metadata, outer_size, outer_stride):
        return mx_tensor(inner_tensors["_mx_packed"], inner_tensors["_mx_scales"],
                         metadata["mx_dtype"], metadata["orig_shape"], metadata["n"],
                         metadata["block"])

    def __reduce_ex__(self, protocol):
        return (_rebuild_mx, (self._mx_packed, self._mx_scales, self._mx_dtype.name,
                              tuple(self._mx_orig_shape), self._mx_n, self._mx_block))

    # ── factory / conversion ─────────────────────────────────────────────────
    @classmethod
    def quantize(cls, x: torch.Tensor, dt, block: int = 128,
                 requires_grad: Optional[bool] = None) -> "mx_tensor":
        """Quantize a float / bf16 tensor (mxtorch.py:6095-6104)."""
        dt = get_mx_dtype(dt)
        packed, scales, n = ops.quantize(x, dt, block)
        return cls(packed, scales, dt, x.shape, n, block)

    def dequantize(self) -> torch.Tensor:
        """fp32 tensor of the original shape (mxtorch.py:6108-6115)."""
        return ops.dequantize(self._mx_packed, self._mx_scales, self._mx_dtype, self._mx_n,
                              self._mx_block, self._mx_orig_shape)

    # ── properties (mxtorch.py:6119-6160) ────────────────────────────────────
    @property
    def shape(self) -> torch.Size:
        return self._mx_orig_shape

    def size(self, dim: Optional[int] = None):
        return self._mx_orig_shape if dim is None else self._mx_orig_shape[dim]

    def dim(self) -> int:
        return len(self._mx_orig_shape)

    def numel(self) -> int:
        return self._mx_n

    @property
    def mx_dtype(self) -> mx_dtype:
        return self._mx_dtype

    @property
    def mx_scales(self) -> torch.Tensor:
        return self._mx_scales

    @property
    def mx_block(self) -> int:
        return self._mx_block

    @property
    def packed(self) -> torch.Tensor:
        return self._mx_packed

    @property
    def nbytes_packed(self) -> int:
        return self._mx_packed.nbytes + self._mx_scales.nbytes

    @property
    def compression_ratio(self) -> float:
        return (self._mx_n * 4) / max(self.nbytes_packed, 1)

    def __repr__(self):
        return (f"mx_tensor({self._mx_dtype.name}, shape={tuple(self._mx_orig_shape)}, "
                f"block={self._mx_block}, device={self._mx_packed.device})")

    __str__ = __repr__

    # ── operators ────────────────────────────────────────────────────────────
    def __matmul__(self, o):
        return _mx_mm(self, o)

    def __rmatmul__(self, o):
        return _mx_mm(o, self)

    def _moved(self, *args, **kwargs) -> "mx_tensor":
        packed = self._mx_packed.to(*args, **kwargs) if args or kwargs else self._mx_packed
        dev = packed.device
        return mx_tensor(packed, self._mx_scales.to(dev), self._mx_dtype, self._mx_orig_shape,
                         self._mx_n, self._mx_block)

    @classmethod
    def __torch_function__(cls, func, types, args=(), kwargs=None):
        kwargs = kwargs or {}
        if func in (torch.matmul, torch.mm, torch.Tensor.matmul, torch.Tensor.mm,
                    torch.Tensor.__matmul__):
            return _mx_mm(args[0], args[1])
        if func in (torch.Tensor.to, torch.Tensor.cuda, torch.Tensor.cpu):
            self = args[0]
            if func is torch.Tensor.cuda:
                dev = args[1] if len(args) > 1 else kwargs.get("device", "cuda")
                return self._moved(torch.device(dev) if not isinstance(dev, int) else
                                   torch.device("cuda", dev))
            if func is torch.Tensor.cpu:
                return self._moved("cpu")
            dev = _device_arg(args[1:], kwargs)
            return self._moved(dev) if dev is not None else self
        if getattr(func, "__name__", "") == "__get__":
            # property reads (.device, .requires_grad, ...) answer from the wrapper
            with torch._C.DisableTorchFunctionSubclass():
                return func(*args, **kwargs)
        if func in (torch.Tensor.detach, torch.Tensor.requires_grad_, torch.Tensor.clone):
            return args[0]
        # everything else: dequantize -> plain torch op (mxtorch.py:7315-7337)
        def unwrap(a):
            return a.dequantize() if isinstance(a, mx_tensor) else a
        with torch._C.DisableTorchFunctionSubclass():
            return func(*tree_map(unwrap, args), **tree_map(unwrap, kwargs))


def _device_arg(args, kwargs):
    cand = list(args) + [kwargs.get("device")]
    for a in cand:
        if isinstance(a, torch.device):
            return a
        if isinstance(a, str) and (a.startswith("cuda") or a == "cpu"):
            return torch.device(a)
        if isinstance(a, int):
            return torch.device("cuda", a)
    return None


def _rebuild_mx(packed, scales, dtype_name, shape, n, block):
    return mx_tensor(packed, scales, get_mx_dtype(dtype_name), shape, n, block)


# ── kernel registry surface (mxtorch.py:5939-6015) ───────────────────────────
@dataclass
class _KernelReg:
    name: str
    op: str
    dtypes: List[str]
    hardware: List[str]
    fn: Callable
    force: str = "auto"
    priority: int = 0

    def matches(self, op, dtype, arch):
        return op == self.op and dtype in self.dtypes and any(h in arch for h in self.hardware)


class _Registry:
    def __init__(self):
        self._kerns: List[_KernelReg] = []

    def add(self, op, dtypes, hardware, force="auto", priority=0):
        def deco(fn):
            self._kerns.append(_KernelReg(fn.__name__, op, list(dtypes), list(hardware), fn,
                                          force, priority))
            return fn
        return deco

    def find(self, op, dtype, arch):
        c = [k for k in self._kerns if k.matches(op, dtype, arch)]
        return max(c, key=lambda k: k.priority) if c else None

    def list_all(self):
        return list(self._kerns)


_REGISTRY = _Registry()
ARCH = "sm_100a"


def register_kernel(op: str, dtypes: List[str], hardware: List[str], force: str = "auto",
                    priority: int = 0):
    """Register a user kernel for an op.  ``force="true"`` on ``torch.matmul``
    routes matching matmuls to the dequantize -> fp32 mm -> requantize path, as
    in the reference (mxtorch.py:6529-6532)."""
    return _REGISTRY.add(op, dtypes, hardware, force, priority)


# ── matmul (mxtorch.py:6508-6549) ────────────────────────────────────────────
def _mm_fallback(a: mx_tensor, b: mx_tensor, out_dt: mx_dtype) -> mx_tensor:
    """dequantize -> fp32 matmul -> requantize (mxtorch.py:6632-6691)."""
    if _STRICT:
        raise RuntimeError(f"[MX_STRICT] full-precision matmul fallback for "
                           f"{a._mx_dtype.name} x {b._mx_dtype.name}")
    r = torch.matmul(a.dequantize(), b.dequantize())
    return mx_tensor.quantize(r, out_dt, a._mx_block)


def _mx_mm(a, b) -> mx_tensor:
    if not isinstance(a, mx_tensor):
        a = mx_tensor.quantize(a, b._mx_dtype, b._mx_block)
    if not isinstance(b, mx_tensor):
        b = mx_tensor.quantize(b, a._mx_dtype, a._mx_block)
    out_dt = optimal_output_dtype("matmul", a._mx_dtype, b._mx_dtype)
    reg = _REGISTRY.find("torch.matmul", a._mx_dtype.name, ARCH)
    if reg is not None and reg.force == "true":
        return _mm_fallback(a, b, out_dt)
    # Every 2-D pair takes the packed GEMM, whatever the kind or variant
    # (mxtorch.py:6534-6540 -> 5563-5573): the reference unpacks both
    # operands' raw codes with A's width, sign-extended (float4d grid
    # indices 8..15 become -8..-1), and runs _qscale_matmul on them.  The
    # kernels take codes of one width for both operands.
    is_2d = len(a._mx_orig_shape) == 2 and len(b._mx_orig_shape) == 2
    if (is_2d and a._mx_dtype.bits == b._mx_dtype.bits and a._mx_dtype.bits in (1, 2, 4, 8)
            and out_dt.bits in (2, 4, 8, 16)):
        return _dispatch_qgemm(a, b, out_dt)
    return _mm_fallback(a, b, out_dt)


def _dispatch_qgemm(a: mx_tensor, b: mx_tensor, out_dt: mx_dtype) -> mx_tensor:
    """Packed GEMM with the reference CPU path's semantics (mxtorch.py:5497-5573)."""
    M, K = a._mx_orig_shape
    K2, N = b._mx_orig_shape
    if K != K2:
        raise ValueError(f"GEMM shape mismatch: {tuple(a._mx_orig_shape)} @ "
                         f"{tuple(b._mx_orig_shape)}")
    block = a._mx_block  # B's scales are viewed [K/block, N] with A's block, as there
    c_packed, c_scales, _ = ops.qgemm(a._mx_packed, a._mx_scales, b._mx_packed, b._mx_scales,
                                      M, K, N, a._mx_dtype.bits, block, out_dt.bits)
    return mx_tensor(c_packed, c_scales, out_dt, torch.Size([M, N]), M * N, block)


def mx_matmul_kmajor(a, b, dtype="int8d", block: int = 128) -> mx_tensor:
    """A @ B with B quantized along K (the k-major mode of the packed matmul).

    ``a`` is an mx_tensor [M, K] or a float tensor (quantized with ``dtype``);
    ``b`` is either a float B [K, N], quantized here as ``B.t()`` so every
    block is one column's K-block, or an mx_tensor already holding B^T
    [N, K].  Each element of B then meets its own block's scale, unlike the
    reference's ``a @ b`` (whose B-scale view, mxtorch.py:1354-1355, pairs
    most elements with another element's scale).  Needs K % block == 0.
    The result is requantized like ``a @ b`` (int16d for int8 x int8)."""
    dt = get_mx_dtype(dtype)
    if not isinstance(a, mx_tensor):
        a = mx_tensor.quantize(a.float(), dt, block)
    if not isinstance(b, mx_tensor):
        b = mx_tensor.quantize(b.float().t().contiguous(), a._mx_dtype, a._mx_block)
    M, K = a._mx_orig_shape
    N, K2 = b._mx_orig_shape
    if K != K2:
        raise ValueError(f"GEMM shape mismatch: {tuple(a._mx_orig_shape)} @ "
                         f"B^T {tuple(b._mx_orig_shape)}")
    if (a._mx_dtype.bits != b._mx_dtype.bits or a._mx_block != b._mx_block
            or not (a._mx_dtype.is_int and b._mx_dtype.is_int)
            or a._mx_dtype.variant != "" or b._mx_dtype.variant != ""
            or a._mx_dtype.bits not in (1, 2, 4, 8)):
        raise NotImplementedError("k-major matmul takes two base int dtypes of one width")
    out_dt = optimal_output_dtype("matmul", a._mx_dtype, b._mx_dtype)
    c_packed, c_scales, _ = ops.qgemm(a._mx_packed, a._mx_scales, b._mx_packed, b._mx_scales,
                                      M, K, N, a._mx_dtype.bits, a._mx_block, out_dt.bits,
                                      b_kmajor=True)
    return mx_tensor(c_packed, c_scales, out_dt, torch.Size([M, N]), M * N, a._mx_block)


def mx_matmul(a: torch.Tensor, b: torch.Tensor, dtype="int4d", block: int = 128) -> mx_tensor:
    """Quantize float operands if needed, then packed matmul (mxtorch.py:10694-10723)."""
    dt = get_mx_dtype(dtype)
    if not isinstance(a, mx_tensor):
        a = mx_tensor.quantize(a.float(), dt, block)
    if not isinstance(b, mx_tensor):
        b = mx_tensor.quantize(b.float(), dt, block)
    return _mx_mm(a, b)
