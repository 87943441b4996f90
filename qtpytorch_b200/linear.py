"""``mx_linear`` and ``to_mx``: weight-only quantized nn.Linear on the mxb kernels.

Mirrors mxtorch.py:7402-7496 (mx_linear) and 9744-9858 (to_mx):
* the weight is stored transposed, ``_mx_weight = quantize(W.t())`` [in, out],
  quantized flat in blocks along ``out``;
* ``forward(x) = fp32(x) @ dequant(W^T)``, fp32 output, computed by the
  split-K GEMV (<= 16 rows) or the tcgen05 GEMM without materialising the
  dequantized weight.

Deliberate differences from the reference:
* the stored bias is applied (the reference replaces it with zeros on every
  forward, mxtorch.py:7434-7436);
* the weight is never replaced by random values when the input's device
  differs (mxtorch.py:7429-7433); the input moves to the weight's device;
* for ``h`` dtypes the output is unrotated along ``out`` -- the rotation
  quantize applied to the rows of W^T -- so ``y = x @ unrotate(dequant)``.
"""
from __future__ import annotations

import re
import warnings
from typing import Dict, List, Optional, Union

import torch
import torch.nn as nn

from . import _lib as L
from . import ops
from .dtypes import get_mx_dtype, mx_dtype
from .tensor import mx_tensor

_SKIP_NAMES = ("float32", "fp32", "float", "float64", "float16", "bfloat16")


class mx_linear(nn.Module):
    """Drop-in replacement for nn.Linear with MX-packed weights."""

    # "parity" keeps fp32-faithful results (error <= 1e-5 of |x| @ |W|);
    # "fast" rounds each dequantized weight to bf16 once
    mode: str = "parity"

    def __init__(self, in_features: int, out_features: int, bias: bool = True,
                 mx_dtype: Optional[mx_dtype] = None, block: int = 128, device=None):
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        self.mx_dtype = get_mx_dtype(mx_dtype or "int4d")
        self.block = block
        self._weight_device = device
        self.register_buffer("_mx_weight", None)
        self.register_buffer("_mx_bias", None)
        self._has_bias = bias

    @classmethod
    def from_linear(cls, linear: nn.Linear, mx_dtype, block: int = 128) -> "mx_linear":
        m = cls.__new__(cls)
        nn.Module.__init__(m)
        m.in_features = linear.in_features
        m.out_features = linear.out_features
        m.mx_dtype = get_mx_dtype(mx_dtype)
        m.block = block
        m._weight_device = None
        m._has_bias = linear.bias is not None
        w = linear.weight.data
        m.register_buffer("_mx_weight", mx_tensor.quantize(w.t(), m.mx_dtype, block))
        if linear.bias is not None:
            m.register_buffer("_mx_bias", mx_tensor.quantize(linear.bias.data, m.mx_dtype, block))
        else:
            m.register_buffer("_mx_bias", None)
        return m

    def _ensure_weight(self, device) -> None:
        # A module built with __init__ gets its weight at the first forward,
        # as in the reference (mxtorch.py:7427-7433).
        if self._mx_weight is None:
            dev = device if device.type == "cuda" else None
            w = torch.randn(self.in_features, self.out_features, device=dev) * 0.01
            self._mx_weight = mx_tensor.quantize(w, self.mx_dtype, self.block)
            if self._has_bias:
                self._mx_bias = mx_tensor.quantize(
                    torch.zeros(self.out_features, device=w.device), self.mx_dtype, self.block)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        self._ensure_weight(x.device)
        w = self._mx_weight
        if isinstance(x, mx_tensor):
            x = x.dequantize()
        lead = x.shape[:-1]
        K, N = self.in_features, self.out_features
        mode = L.MODE_FAST if self.mode == "fast" else L.MODE_PARITY
        y = ops.linear_wonly(x.reshape(-1, K), w._mx_packed, w._mx_scales, K, N, w._mx_dtype,
                             w._mx_block, mode)
        if w._mx_dtype.is_hadamard:
            y = ops.hadamard_rows(y, w._mx_dtype.hadamard_seed, inverse=True)
        if self._mx_bias is not None:
            y = y + self._mx_bias.dequantize()
        return y.reshape(*lead, N)

    @property
    def weight(self):
        return None if self._mx_weight is None else self._mx_weight.dequantize().t()

    @property
    def bias(self):
        return None if self._mx_bias is None else self._mx_bias.dequantize()

    def _apply(self, fn, recurse=True):
        # keep the packed buffers packed when the module moves devices
        for key in ("_mx_weight", "_mx_bias"):
            t = self._buffers.get(key)
            if isinstance(t, mx_tensor):
                probe = fn(torch.empty(0, device=t._mx_packed.device))
                self._buffers[key] = t._moved(probe.device)
        return self

    def extra_repr(self):
        return (f"in={self.in_features}, out={self.out_features}, "
                f"dtype={self.mx_dtype.name}, bias={self._mx_bias is not None}")


def _replace_module(parent: nn.Module, name: str, module: nn.Module, dt: mx_dtype,
                    block: int) -> bool:
    """Swap nn.Linear for mx_linear (mxtorch.py:7977-7989).  Other module
    kinds are not on the B200 path and stay as they are."""
    if isinstance(module, nn.Linear):
        setattr(parent, name, mx_linear.from_linear(module, dt, block))
        return True
    return False


def to_mx(model: nn.Module, dtype: Union[str, Dict[str, str], mx_dtype] = "int4d",
          block_size: int = 128, low_mem: bool = False, layer_batch_size: int = 4,
          skip_patterns: Optional[List[str]] = None) -> nn.Module:
    """Quantize every nn.Linear of ``model`` in place (mxtorch.py:9744-9858).

    ``dtype`` is a dtype name / mx_dtype, or a dict of regex -> dtype matched
    against module names and class names (first match wins).
    """
    if isinstance(dtype, mx_dtype):
        dtype = dtype.name
    elif getattr(dtype, "_mx", None) is not None:
        dtype = dtype._mx.name
    if isinstance(dtype, str):
        dtype_map = {".*": dtype}
    elif isinstance(dtype, dict):
        dtype_map = {p: (v.name if isinstance(v, mx_dtype) else v) for p, v in dtype.items()}
    else:
        raise TypeError(f"dtype must be str, dict or mx_dtype, got {type(dtype)}")
    skip = skip_patterns or []
    named = list(model.named_modules())
    for full_name, module in named:
        if not isinstance(module, nn.Linear):
            continue
        if any(re.search(p, full_name) for p in skip):
            continue
        target = None
        for pat, dt_name in dtype_map.items():
            if re.search(pat, full_name) or re.search(pat, type(module).__name__):
                target = dt_name
                break
        if target is None or target in _SKIP_NAMES:
            continue
        try:
            dt = get_mx_dtype(target)
        except ValueError:
            warnings.warn(f"Unknown dtype {target!r} for {full_name}, skipping.")
            continue
        for pname, pmod in named:
            done = False
            for cname, cmod in pmod.named_children():
                if cmod is module:
                    _replace_module(pmod, cname, module, dt, block_size)
                    done = True
                    break
            if done:
                break
    return model
