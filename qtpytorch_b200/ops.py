"""Tensor-level wrappers of the mxb C ABI (no autograd, no dispatch).

Each function takes and returns torch tensors on a CUDA device, allocates
outputs and workspaces with torch, and launches on the current stream.
CPU inputs are copied to the current CUDA device first; nothing here
computes on the CPU.
"""
from __future__ import annotations

import math
from typing import Optional, Tuple

import torch

from . import _lib as L
from .dtypes import KERNEL_BITS, get_mx_dtype, mx_dtype
from .hadamard import device_signs


def _device_of(x: torch.Tensor) -> torch.device:
    if x.is_cuda:
        return x.device
    if not torch.cuda.is_available():
        raise L.MxbError("qtpytorch_b200 needs a CUDA device (B200, sm_100a)")
    return torch.device("cuda", torch.cuda.current_device())


def kernel_dtype_ok(dt: mx_dtype) -> bool:
    if dt.variant not in ("", "h"):
        return False
    if dt.is_float:
        return dt.bits == 4
    return dt.bits in KERNEL_BITS


def _kind(dt: mx_dtype) -> int:
    return L.KIND_FLOAT if dt.is_float else L.KIND_INT


def _check_dtype(dt: mx_dtype) -> None:
    if not kernel_dtype_ok(dt):
        raise NotImplementedError(
            f"{dt.name}: the B200 kernels cover int1/int2/int4/int8 'd'/'u' and float4, "
            f"base and 'h' variants")


def row_len_of(shape) -> int:
    n = 1
    for s in shape:
        n *= int(s)
    if len(shape) >= 2:
        return int(shape[-1])
    return max(n, 1)


def quantize(x: torch.Tensor, dt, block: int = 128,
             out: Optional[Tuple[torch.Tensor, torch.Tensor]] = None
             ) -> Tuple[torch.Tensor, torch.Tensor, int]:
    """(packed int8, scales fp32 [nb], n): mxtorch ``quantize`` (mxtorch.py:1684-1763).

    ``out``: (packed, scales) contiguous device buffers to write into (at
    least the packed bytes and the scale count of this call)."""
    dt = get_mx_dtype(dt)
    _check_dtype(dt)
    if block <= 0:
        raise ValueError("block must be positive")
    dev = _device_of(x)
    x = x.detach()
    if x.dtype not in (torch.float32, torch.bfloat16):
        x = x.float()
    x = x.to(dev).contiguous()
    n = x.numel()
    nb = -(-n // block)
    lib = L.load()
    nbytes = lib.mxb_packed_bytes(n, dt.bits, block)
    if out is None:
        packed = torch.empty(nbytes, dtype=torch.int8, device=dev)
        scales = torch.empty(nb, dtype=torch.float32, device=dev)
    else:
        packed, scales = out
        if (packed.device != dev or scales.device != dev or not packed.is_contiguous()
                or not scales.is_contiguous() or packed.numel() * packed.element_size() < nbytes
                or scales.numel() < nb or scales.dtype != torch.float32):
            raise ValueError("quantize: out buffers too small, not contiguous or on another device")
    if n == 0:
        return packed, scales, 0
    row_len = row_len_of(x.shape)
    variant = L.VAR_H if dt.is_hadamard else L.VAR_BASE
    signs = device_signs(row_len, dt.hadamard_seed, dev) if dt.is_hadamard else None
    kind = _kind(dt)
    in_t = L.BF16 if x.dtype == torch.bfloat16 else L.F32
    wsb = lib.mxb_quantize_workspace_size(n, row_len, dt.bits, kind, variant, block)
    ws = L.workspace(wsb, dev)
    with torch.cuda.device(dev):
        rc = lib.mxb_quantize(L.ptr(x), in_t, n, row_len, dt.bits, kind, variant, block,
                              L.ptr(signs), L.ptr(packed), L.ptr(scales), L.ptr(ws), wsb,
                              L.stream_of(dev))
    L.check(rc, f"mxb_quantize({dt.name}, n={n}, block={block})")
    return packed, scales, n


def dequantize(packed: torch.Tensor, scales: torch.Tensor, dt, n: int, block: int,
               shape=None) -> torch.Tensor:
    """fp32 tensor of ``shape`` (flat if None): mxtorch ``_dequant`` (mxtorch.py:1530-1597).

    For ``h`` dtypes the inverse rotation runs along the last dim of ``shape``.
    """
    dt = get_mx_dtype(dt)
    if not (kernel_dtype_ok(dt) or (dt.is_int and dt.bits == 16 and dt.variant == "")):
        raise NotImplementedError(f"dequantize of {dt.name} is not on the B200 path")
    L.require_cuda(packed, "dequantize")
    dev = packed.device
    shape = tuple(shape) if shape is not None else (n,)
    out = torch.empty(n, dtype=torch.float32, device=dev)
    if n == 0:
        return out.reshape(shape)
    row_len = row_len_of(shape)
    variant = L.VAR_H if dt.is_hadamard else L.VAR_BASE
    signs = device_signs(row_len, dt.hadamard_seed, dev) if dt.is_hadamard else None
    lib = L.load()
    with torch.cuda.device(dev):
        rc = lib.mxb_dequantize(L.ptr(packed.contiguous()), L.ptr(scales.contiguous()), n,
                                row_len, dt.bits, _kind(dt), variant, block, L.ptr(signs),
                                L.ptr(out), L.stream_of(dev))
    L.check(rc, f"mxb_dequantize({dt.name}, n={n})")
    return out.reshape(shape)


def hadamard_rows(y: torch.Tensor, seed: Optional[int], inverse: bool) -> torch.Tensor:
    """Randomized WHT along the last dim of a fp32 CUDA tensor (in a new tensor).
    ``seed`` None: unit signs (the plain WHT / sqrt(n))."""
    L.require_cuda(y, "hadamard_rows")
    y = y.float().contiguous()
    d = y.shape[-1]
    rows = y.numel() // max(d, 1)
    out = torch.empty_like(y)
    if seed is None:
        from .hadamard import pow2ceil
        signs = torch.ones(pow2ceil(d), dtype=torch.float32, device=y.device)
    else:
        signs = device_signs(d, seed, y.device)
    with torch.cuda.device(y.device):
        rc = L.load().mxb_hadamard_rows(L.ptr(y), rows, d, L.ptr(signs), int(inverse),
                                        L.ptr(out), L.stream_of(y.device))
    L.check(rc, "mxb_hadamard_rows")
    return out


def hadamard_cross(t: torch.Tensor, M: int, cols: int, G: int, seed: int) -> torch.Tensor:
    """[M, G*cols] fp32 from the gathered [G, M, cols] per-shard transforms
    t_g = WHT(y_g)/sqrt(cols): the G-point cross-shard stage, / sqrt(G), times
    the signs of the full row (mxb_hadamard_cross)."""
    L.require_cuda(t, "hadamard_cross")
    t = t.float().contiguous()
    out = torch.empty(M, G * cols, dtype=torch.float32, device=t.device)
    signs = device_signs(G * cols, seed, t.device)
    with torch.cuda.device(t.device):
        rc = L.load().mxb_hadamard_cross(L.ptr(t), M, cols, G, L.ptr(signs), L.ptr(out),
                                         L.stream_of(t.device))
    L.check(rc, f"mxb_hadamard_cross(M={M}, L={cols}, G={G})")
    return out


def qgemm(a_packed, a_scales, b_packed, b_scales, M: int, K: int, N: int, bits: int,
          block: int, out_bits: int, want_f32: bool = False, b_kmajor: bool = False):
    """Packed integer matmul (mxtorch.py:5497-5573 CPU branch, bit-exact).

    Returns (c_packed, c_scales, c_f32 or None); c_packed is int32 words for
    16-bit codes, int8 bytes otherwise.  out_bits 32: (None, None, c_f32),
    the fp32 C without requantization.  ``b_kmajor``: b_packed / b_scales
    hold B^T [N, K] quantized along K (each element with its own block's
    scale), computed by ``mxb_qgemm_kmajor``.
    """
    L.require_cuda(a_packed, "qgemm")
    dev = a_packed.device
    lib = L.load()
    nb = -(-(M * N) // block)
    if out_bits == 32:  # the fp32 C alone, no requantization
        c_packed = c_scales = None
        want_f32 = True
    elif out_bits == 16:
        c_packed = torch.empty(lib.mxb_packed_bytes(M * N, 16, block) // 4, dtype=torch.int32,
                               device=dev)
    else:
        c_packed = torch.empty(lib.mxb_packed_bytes(M * N, out_bits, block), dtype=torch.int8,
                               device=dev)
    if out_bits != 32:
        c_scales = torch.empty(nb, dtype=torch.float32, device=dev)
    c_f32 = torch.empty(M, N, dtype=torch.float32, device=dev) if want_f32 else None
    wsf = lib.mxb_qgemm_kmajor_workspace_size if b_kmajor else lib.mxb_qgemm_workspace_size
    fn = lib.mxb_qgemm_kmajor if b_kmajor else lib.mxb_qgemm
    wsb = wsf(M, K, N, bits, block)
    ws = L.workspace(wsb, dev)
    a_packed, b_packed = a_packed.contiguous(), b_packed.to(dev).contiguous()
    a_scales, b_scales = a_scales.contiguous(), b_scales.to(dev).contiguous()
    with torch.cuda.device(dev):
        rc = fn(L.ptr(a_packed), L.ptr(a_scales), a_scales.numel(),
                L.ptr(b_packed), L.ptr(b_scales), b_scales.numel(), M, K, N, bits,
                block, out_bits, L.ptr(c_packed), L.ptr(c_scales), L.ptr(c_f32),
                L.ptr(ws), wsb, L.stream_of(dev))
    name = "mxb_qgemm_kmajor" if b_kmajor else "mxb_qgemm"
    L.check(rc, f"{name}({M}x{K}x{N}, bits={bits})")
    return c_packed, c_scales, c_f32


def linear_wonly(x: torch.Tensor, w_packed: torch.Tensor, w_scales: torch.Tensor, K: int,
                 N: int, dt, block: int, mode: int = L.MODE_PARITY,
                 out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """y[M, N] fp32 = fp32(x[M, K]) @ dequant(W^T) (mxtorch.py:7454-7473)."""
    dt = get_mx_dtype(dt)
    _check_dtype(dt)
    L.require_cuda(w_packed, "linear_wonly")
    dev = w_packed.device
    if x.dtype not in (torch.float32, torch.bfloat16):
        x = x.float()
    x = x.to(dev).contiguous()
    M = x.numel() // K
    y = out if out is not None else torch.empty(M, N, dtype=torch.float32, device=dev)
    lib = L.load()
    wsb = lib.mxb_linear_wonly_workspace_size(M, K, N, dt.bits, _kind(dt), block, mode)
    ws = L.workspace(wsb, dev)
    in_t = L.BF16 if x.dtype == torch.bfloat16 else L.F32
    with torch.cuda.device(dev):
        rc = lib.mxb_linear_wonly(L.ptr(x), in_t, M, K, L.ptr(w_packed), L.ptr(w_scales), N,
                                  dt.bits, _kind(dt), block, mode, L.ptr(y), L.ptr(ws), wsb,
                                  L.stream_of(dev))
    L.check(rc, f"mxb_linear_wonly({M}x{K}x{N}, {dt.name})")
    return y


def linear_wonly_kmajor(x: torch.Tensor, w_packed: torch.Tensor, w_scales: torch.Tensor, K: int,
                        N: int, dt, block: int, mode: int = L.MODE_PARITY) -> torch.Tensor:
    """y[M, N] fp32 = x[M, K] @ dequant(W)^T for W [N, K] quantized flat (its
    blocks run along K): the matmul of mx_dynamic_linear.forward
    (mxtorch.py:8947-8978) without a dequantized weight.  Base dtypes."""
    dt = get_mx_dtype(dt)
    _check_dtype(dt)
    if dt.is_hadamard:
        raise NotImplementedError("linear_wonly_kmajor takes base dtypes (rotate x for 'h')")
    L.require_cuda(w_packed, "linear_wonly_kmajor")
    dev = w_packed.device
    if x.dtype not in (torch.float32, torch.bfloat16):
        x = x.float()
    x = x.to(dev).contiguous()
    M = x.numel() // K
    y = torch.empty(M, N, dtype=torch.float32, device=dev)
    in_t = L.BF16 if x.dtype == torch.bfloat16 else L.F32
    with torch.cuda.device(dev):
        rc = L.load().mxb_linear_wonly_kmajor(L.ptr(x), in_t, M, K, L.ptr(w_packed),
                                              L.ptr(w_scales.contiguous()), N, dt.bits,
                                              _kind(dt), block, mode, L.ptr(y), L.stream_of(dev))
    L.check(rc, f"mxb_linear_wonly_kmajor({M}x{K}x{N}, {dt.name})")
    return y


def dynamic_quantize(x: torch.Tensor, bits: int, block: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """(packed, scales) of ``mxb_dynamic_quantize``: flat blocks of any
    length, scale = max(amax, 1e-12) / max_int, codes = rint(x / scale)
    (mxtorch.py:2665-2712).  packed is int32 words for 16-bit codes."""
    dev = _device_of(x)
    x = x.detach()
    if x.dtype not in (torch.float32, torch.bfloat16):
        x = x.float()
    x = x.to(dev).contiguous()
    n = x.numel()
    lib = L.load()
    nbytes = lib.mxb_packed_bytes(n, bits, block)
    if bits == 16:
        packed = torch.empty(nbytes // 4, dtype=torch.int32, device=dev)
    else:
        packed = torch.empty(nbytes, dtype=torch.int8, device=dev)
    scales = torch.empty(-(-n // block), dtype=torch.float32, device=dev)
    if n == 0:
        return packed, scales
    wsb = lib.mxb_dynamic_quantize_workspace_size(n, block)
    ws = L.workspace(wsb, dev)
    in_t = L.BF16 if x.dtype == torch.bfloat16 else L.F32
    with torch.cuda.device(dev):
        rc = lib.mxb_dynamic_quantize(L.ptr(x), in_t, n, block, bits, L.ptr(packed),
                                      L.ptr(scales), L.ptr(ws), wsb, L.stream_of(dev))
    L.check(rc, f"mxb_dynamic_quantize(n={n}, block={block}, bits={bits})")
    return packed, scales


def dequantize_relu(packed: torch.Tensor, scales: torch.Tensor, dt, n: int,
                    block: int) -> torch.Tensor:
    """relu(dequantize) in one pass (mxtorch.py:3441-3456, 4012-4074), fp32 [n]."""
    dt = get_mx_dtype(dt)
    if dt.variant != "":
        raise NotImplementedError("dequantize_relu takes base dtypes")
    L.require_cuda(packed, "dequantize_relu")
    dev = packed.device
    out = torch.empty(n, dtype=torch.float32, device=dev)
    if n == 0:
        return out
    lib = L.load()
    with torch.cuda.device(dev):
        rc = lib.mxb_dequantize_relu(L.ptr(packed), L.ptr(scales.contiguous()), n, dt.bits,
                                     _kind(dt), block, L.ptr(out), L.stream_of(dev))
    L.check(rc, f"mxb_dequantize_relu({dt.name}, n={n})")
    return out


def dequantize_silu_mul(gp: torch.Tensor, gs: torch.Tensor, up: torch.Tensor, us: torch.Tensor,
                        dt, n: int, block: int) -> torch.Tensor:
    """SiLU(dequant(gate)) * dequant(up) in one pass (mxtorch.py:3459-3479), fp32 [n]."""
    dt = get_mx_dtype(dt)
    if dt.variant != "":
        raise NotImplementedError("dequantize_silu_mul takes base dtypes")
    L.require_cuda(gp, "dequantize_silu_mul")
    dev = gp.device
    out = torch.empty(n, dtype=torch.float32, device=dev)
    if n == 0:
        return out
    lib = L.load()
    with torch.cuda.device(dev):
        rc = lib.mxb_dequantize_silu_mul(L.ptr(gp), L.ptr(gs.contiguous()), L.ptr(up.to(dev)),
                                         L.ptr(us.to(dev).contiguous()), n, dt.bits, _kind(dt),
                                         block, L.ptr(out), L.stream_of(dev))
    L.check(rc, f"mxb_dequantize_silu_mul({dt.name}, n={n})")
    return out
