"""Dequantize-fused activations after the packed matmul.

Mirrors of mxtorch's ``fused_linear_relu`` (mxtorch.py:4012-4074) and
``fused_silu_and_mul`` (4077-4109).  The activation runs inside the
dequantize kernel (``mxb_dequantize_relu`` / ``mxb_dequantize_silu_mul``), so
no fp32 copy of the pre-activation is written.  The reference's own GPU
branch of ``fused_linear_relu`` reads the int16d matmul result as int8 codes;
its CPU branch, ``relu(y.dequantize())``, is the formula kept here, for every
output width.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.nn.functional as F

from . import ops
from .dtypes import get_mx_dtype
from .tensor import _mx_mm, mx_tensor


def _as_2d(x: mx_tensor, K: int) -> mx_tensor:
    # the packed layout is flat, so a [.., K] tensor is the same bytes as [M, K]
    return mx_tensor(x._mx_packed, x._mx_scales, x._mx_dtype, (x._mx_n // K, K), x._mx_n,
                     x._mx_block)


def fused_linear_relu(x: torch.Tensor, weight, bias: Optional[torch.Tensor] = None,
                      block: int = 128, mx_dtype=None) -> torch.Tensor:
    """relu(x @ W) (+ bias) with the matmul in packed precision
    (mxtorch.py:4012-4074).  ``weight``: an mx_tensor [in, out] (as
    ``mx_linear._mx_weight``) or a float [out, in] (as ``nn.Linear.weight``,
    quantized transposed with ``mx_dtype``, default int8d)."""
    if isinstance(weight, mx_tensor):
        w_mx = weight
        dtype = w_mx._mx_dtype
        out_features = w_mx.shape[-1]
    else:
        dtype = get_mx_dtype(mx_dtype or "int8d")
        w_mx = mx_tensor.quantize(weight.float().t(), dtype, block)
        out_features = weight.shape[0]
    K = x.shape[-1]
    lead = x.shape[:-1]
    if isinstance(x, mx_tensor):
        x_mx = _as_2d(x, K)
    else:
        x_mx = mx_tensor.quantize(x.float().reshape(-1, K), dtype, block)
    y = _mx_mm(x_mx, w_mx)
    out = ops.dequantize_relu(y._mx_packed, y._mx_scales, y._mx_dtype, y._mx_n, y._mx_block)
    out = out.reshape(*lead, out_features)
    if bias is not None:
        b = bias.dequantize() if isinstance(bias, mx_tensor) else bias
        out = out + b.to(out.device)
    return out


def fused_silu_and_mul(gate, up) -> torch.Tensor:
    """SiLU(gate) * up, the SwiGLU activation (mxtorch.py:4077-4109).  Two
    packed operands of one base dtype, block and length run in one kernel;
    anything else is dequantized first."""
    if (isinstance(gate, mx_tensor) and isinstance(up, mx_tensor)
            and gate._mx_dtype.name == up._mx_dtype.name and gate._mx_dtype.variant == ""
            and gate._mx_n == up._mx_n and gate._mx_block == up._mx_block):
        out = ops.dequantize_silu_mul(gate._mx_packed, gate._mx_scales, up._mx_packed,
                                      up._mx_scales, gate._mx_dtype, gate._mx_n, gate._mx_block)
        return out.reshape(gate._mx_orig_shape)
    g = gate.dequantize() if isinstance(gate, mx_tensor) else gate
    u = up.dequantize() if isinstance(up, mx_tensor) else up
    return F.silu(g) * u
