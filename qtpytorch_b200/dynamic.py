"""Dynamic activation quantize and the full-int8 linear.

Mirrors of mxtorch's ``dynamic_quantize`` (mxtorch.py:2665-2712),
``fused_int8_linear`` (3910-3960) and ``mx_dynamic_linear`` (8870-8978).

- ``dynamic_quantize``: one CUDA kernel launch (``mxb_dynamic_quantize``)
  over flat blocks of any length; codes and scales bit-identical to the
  reference's CPU arithmetic.
- ``fused_int8_linear``: the packed operands go straight into the k-major
  integer GEMM (tcgen05 ``kind::i8`` where the shape allows), which returns
  the fp32 sum over K-blocks of sx * sw * (integer dot product); the
  reference's CPU branch is F.linear of the dequantized operands, so the
  result agrees to fp32 rounding.  A per-token x (one scale per row) meets
  the weight's K-blocks by repeating its scale per block.
- ``mx_dynamic_linear``: the reference quantizes the activations but its
  output uses the fp32 activations and the dequantized weight (8960-8967),
  so here the packed [out, in] weight goes straight into the K-major
  weight-only kernel (``mxb_linear_wonly_kmajor``) with the activations as
  given; the activation codes, which nothing reads, are not computed.
"""
from __future__ import annotations

from typing import Optional, Union

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import ops
from .dtypes import get_mx_dtype, mx_dtype
from .tensor import mx_tensor

_GRANULARITIES = ("per_token", "per_channel", "per_tensor", "per_block")


def dynamic_quantize(x: torch.Tensor, dtype: Union[str, mx_dtype] = "int8d",
                     granularity: str = "per_token", block: int = 64) -> mx_tensor:
    """Runtime quantize with scales from the input (mxtorch.py:2665-2712).

    "per_token": one scale per row of the last dim; "per_channel": one per
    column of x.reshape(shape[0], -1) (int8 codes only); "per_tensor": one
    for the whole tensor; "per_block": ``mx_tensor.quantize(x, dtype, block)``.
    """
    dt = get_mx_dtype(dtype)
    if granularity not in _GRANULARITIES:
        raise ValueError(f"granularity must be one of {_GRANULARITIES}, got {granularity!r}")
    if granularity == "per_block":
        return mx_tensor.quantize(x.float(), dt, block)
    if not dt.is_int or dt.variant != "" or dt.bits not in (2, 4, 8, 16):
        raise NotImplementedError(f"dynamic_quantize covers base int dtypes of 2-16 bits, "
                                  f"not {dt.name}")
    shape = x.shape
    if granularity == "per_token":
        blk = shape[-1] if len(shape) else 1
        packed, scales = ops.dynamic_quantize(x, dt.bits, blk)
    elif granularity == "per_tensor":
        blk = max(x.numel(), 1)
        packed, scales = ops.dynamic_quantize(x, dt.bits, blk)
    else:  # per_channel: quantize the columns as rows, then put the codes back
        if dt.bits != 8:
            raise NotImplementedError("per_channel dynamic_quantize covers int8 codes")
        x2 = x.reshape(shape[0], -1)
        blk = shape[0]
        packed_t, scales = ops.dynamic_quantize(x2.t().contiguous(), 8, blk)
        packed = packed_t.view(x2.shape[1], x2.shape[0]).t().contiguous().view(-1)
    return mx_tensor(packed, scales, dt, shape, x.numel(), blk)


def _kblock_scales(t: mx_tensor, rows: int, K: int, block: int) -> torch.Tensor:
    """Scales of a [rows, K] tensor as [rows, K / block] (its own block a
    multiple of ``block``, one K-block of ``block`` per entry)."""
    own = t._mx_block
    s = t._mx_scales[: rows * (K // own)].view(rows, K // own)
    if own != block:
        s = s.repeat_interleave(own // block, dim=1)
    return s.contiguous().view(-1)


def fused_int8_linear(x: mx_tensor, weight: mx_tensor, bias: Optional[torch.Tensor] = None,
                      block: int = 128) -> torch.Tensor:
    """Full-int8 linear: out[M, N] fp32 = x[M, K] @ weight[N, K]^T + bias
    (mxtorch.py:3910-3960), both operands packed, no dequantized copy.

    Runs the k-major integer GEMM when x and weight hold base int codes of one
    width whose scale blocks nest (one a multiple of the other, both dividing
    K); otherwise x is dequantized (CUDA kernel) and meets the packed weight
    in the K-major weight-only kernel, the reference's CPU formula
    F.linear(dequant(x), dequant(W)) without a dequantized weight."""
    if not isinstance(x, mx_tensor) or not isinstance(weight, mx_tensor):
        raise TypeError("fused_int8_linear takes two mx_tensors")
    K = x._mx_orig_shape[-1] if len(x._mx_orig_shape) >= 2 else x._mx_block
    M = x._mx_n // K
    N = weight._mx_n // K
    xd, wd = x._mx_dtype, weight._mx_dtype
    bx, bw = x._mx_block, weight._mx_block
    kb = min(bx, bw)
    direct = (xd.is_int and wd.is_int and xd.variant == "" and wd.variant == ""
              and xd.bits == wd.bits and xd.bits in (1, 2, 4, 8)
              and max(bx, bw) % kb == 0 and K % bx == 0 and K % bw == 0
              and x._mx_n == M * K and weight._mx_n == N * K)
    if direct:
        sx = _kblock_scales(x, M, K, kb)
        sw = _kblock_scales(weight, N, K, kb)
        _, _, out = ops.qgemm(x._mx_packed, sx, weight._mx_packed, sw, M, K, N, xd.bits, kb,
                              32, b_kmajor=True)
    elif ops.kernel_dtype_ok(wd) and weight._mx_n == N * K:
        # the dequantized x against the packed weight, read K-major as stored
        out = _kmajor_linear(x.dequantize().reshape(M, K), weight, K, N)
    else:  # weight dtype outside the kernels: the reference's formula
        out = F.linear(x.dequantize().reshape(M, K), weight.dequantize().reshape(N, K))
    if bias is not None:
        out = out + bias.to(out.device).float()
    return out


def _kmajor_linear(tokens: torch.Tensor, w: mx_tensor, K: int, N: int) -> torch.Tensor:
    """tokens [M, K] @ dequant(W)^T for W [N, K] quantized flat, on the
    K-major weight-only kernel.  An ``h`` weight (rotated along K) meets the
    tokens rotated the same way: x @ unrotate(D)^T = rotate(x) @ D^T."""
    dt = w._mx_dtype
    if dt.is_hadamard:
        tokens = ops.hadamard_rows(tokens.float(), dt.hadamard_seed, inverse=False)
        dt = dt.base
    return ops.linear_wonly_kmajor(tokens, w._mx_packed, w._mx_scales, K, N, dt, w._mx_block)


class mx_dynamic_linear(nn.Module):
    """Static MX weight, per-token dynamic activations (mxtorch.py:8870-8978).

    The weight is ``mx_tensor.quantize(linear.weight, weight_dtype, block)``,
    [out, in] quantized along ``in``, as in the reference."""

    def __init__(self, in_features: int, out_features: int, weight_dtype=None,
                 act_dtype=None, bias: bool = True, weight_block: int = 128):
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        self.weight_dtype = get_mx_dtype(weight_dtype or "int4d")
        self.act_dtype = get_mx_dtype(act_dtype or "int8d")
        self.weight_block = weight_block
        self.register_buffer("weight", None)
        self.register_buffer("bias", None)

    @classmethod
    def from_linear(cls, linear: nn.Linear, weight_dtype="int4d", act_dtype="int8d",
                    weight_block: int = 128) -> "mx_dynamic_linear":
        m = cls(linear.in_features, linear.out_features, weight_dtype, act_dtype,
                linear.bias is not None, weight_block)
        dev = linear.weight.device if linear.weight.is_cuda else torch.device("cuda")
        m.weight = mx_tensor.quantize(linear.weight.data.to(dev), m.weight_dtype, weight_block)
        if linear.bias is not None:
            m.bias = linear.bias.data.detach().clone().to(dev)
        return m

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """fp32(x) @ dequant(W)^T + bias (mxtorch.py:8947-8978) on the K-major
        weight-only kernel: the packed [out, in] weight is read as stored.
        A bf16 x is passed as is (its fp32 value is exact in bf16); an ``h``
        weight, rotated along ``in``, meets x rotated the same way, since
        x @ unrotate(D)^T = rotate(x) @ D^T."""
        x_f = x.dequantize() if isinstance(x, mx_tensor) else x
        if x_f.dtype not in (torch.float32, torch.bfloat16):
            x_f = x_f.float()
        w = self.weight
        if not isinstance(w, mx_tensor):
            w = mx_tensor.quantize(w, self.weight_dtype, self.weight_block)
        K, N = self.in_features, self.out_features
        tokens = x_f.reshape(-1, K).to(w._mx_packed.device)
        if ops.kernel_dtype_ok(w._mx_dtype):
            out = _kmajor_linear(tokens, w, K, N)
        else:  # weight dtype outside the kernels: the reference's formula
            out = tokens.float() @ w.dequantize().reshape(N, K).t()
        out = out.reshape(*x_f.shape[:-1], N)
        if self.bias is not None:
            out = out + self.bias
        return out

    def extra_repr(self):
        return (f"in={self.in_features}, out={self.out_features}, "
                f"w={self.weight_dtype.name}, act={self.act_dtype.name}")
