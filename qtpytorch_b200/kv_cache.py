"""Quantized KV cache (mxtorch ``kv_cache_quantizer``, mxtorch.py:2998-3119).

The reference keeps one mx_tensor per generated step in a Python list.  Here
the steps live in device ring buffers, one slot per step, grown by doubling
up to ``max_seq_len``:

- K: packed codes [cap, BH * D * bits / 8] and scales [cap, BH], block =
  head_dim (one scale per head row, as the reference's
  ``mx_tensor.quantize(k.reshape(-1, D), dtype, D)``);
- V: the same, of v - rowmin(v) when ``asymmetric_v``, with the row minima
  (the zero points) in [cap, BH] fp32.

``append_kv`` quantizes the step straight into its slot (one quantize launch
per tensor); at ``max_seq_len`` the oldest slot is overwritten, as the
reference's ``pop(0)``.  ``get`` dequantizes all live slots with one launch
per tensor and returns [B, H, T, D] fp32, bit-identical to the reference's
stack of per-step dequantizes (plus the fp32 zero-point add for V) for the
base dtypes.  ``h`` dtypes rotate and unrotate each head row (the
framework's convention for every quantized tensor of 2 or more dims).
"""
from __future__ import annotations

from typing import List, Tuple, Union

import torch

from . import _lib as L
from . import ops
from .dtypes import get_mx_dtype, mx_dtype
from .tensor import mx_tensor


class _Ring:
    """Packed codes + scales of one tensor stream, one slot per step."""

    def __init__(self, rows: int, D: int, dt: mx_dtype, cap: int, device, with_zp: bool):
        self.rows, self.D, self.dt = rows, D, dt
        self.row_bytes = L.load().mxb_packed_bytes(rows * D, dt.bits, D)
        self.packed = torch.empty(cap, self.row_bytes, dtype=torch.int8, device=device)
        self.scales = torch.empty(cap, rows, dtype=torch.float32, device=device)
        self.zp = torch.empty(cap, rows, dtype=torch.float32, device=device) if with_zp else None

    @property
    def cap(self) -> int:
        return self.packed.shape[0]

    def grow(self, cap: int, live: int) -> None:
        # only called while the ring has not wrapped: slots 0..live-1 in order
        for name in ("packed", "scales", "zp"):
            t = getattr(self, name)
            if t is None:
                continue
            n = torch.empty((cap,) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
            n[:live].copy_(t[:live])
            setattr(self, name, n)

    def put(self, slot: int, x: torch.Tensor, block: int) -> None:
        ops.quantize(x, self.dt, block, out=(self.packed[slot], self.scales[slot]))

    def step(self, slot: int) -> mx_tensor:
        return mx_tensor(self.packed[slot], self.scales[slot], self.dt, (self.rows, self.D),
                         self.rows * self.D, self.D)

    def dequant(self, order: torch.Tensor) -> torch.Tensor:
        """[rows, T, D] fp32 of the slots in ``order``."""
        T = order.numel()
        p = self.packed.index_select(0, order).view(-1)
        s = self.scales.index_select(0, order).view(-1)
        flat = ops.dequantize(p, s, self.dt, T * self.rows * self.D, self.D,
                              shape=(T * self.rows, self.D))
        return flat.view(T, self.rows, self.D).transpose(0, 1)


class kv_cache_quantizer:
    """Quantized KV cache for long-context decoding (mxtorch.py:2998-3119).

    cache = kv_cache_quantizer(n_heads=32, head_dim=128, dtype="int8d")
    cache.append_kv(k_new, v_new)        # k/v: [B, H, 1, D] or [B, 1, H, D]
    k_hist, v_hist = cache.get()         # [B, H, T, D] fp32
    """

    _INITIAL_CAP = 64

    def __init__(self, n_heads: int, head_dim: int, dtype: Union[str, mx_dtype] = "int8d",
                 max_seq_len: int = 32768, asymmetric_v: bool = True):
        self.n_heads = n_heads
        self.head_dim = head_dim
        self.dtype = get_mx_dtype(dtype) if isinstance(dtype, str) else dtype
        self.max_seq_len = max_seq_len
        self.asymmetric_v = asymmetric_v
        self._k = self._v = None
        self._head = 0  # slot of the oldest live step
        self._len = 0

    def append_kv(self, k: torch.Tensor, v: torch.Tensor) -> None:
        """Quantize and store one step's K and V slices."""
        D = self.head_dim
        k_f = k.float().reshape(-1, D)
        v_f = v.float().reshape(-1, D)
        if not k_f.is_cuda:
            raise L.MxbError("kv_cache_quantizer: the mxb kernels run on CUDA tensors only")
        rows = k_f.shape[0]
        if self._k is None:
            cap = min(self._INITIAL_CAP, self.max_seq_len)
            self._k = _Ring(rows, D, self.dtype, cap, k_f.device, False)
            self._v = _Ring(rows, D, self.dtype, cap, k_f.device, self.asymmetric_v)
        elif rows != self._k.rows:
            raise ValueError(f"append_kv: {rows} rows of head_dim, the cache holds {self._k.rows}")
        if self._len >= self.max_seq_len:  # evict the oldest step
            self._head = (self._head + 1) % self._k.cap
            self._len -= 1
        elif self._len == self._k.cap:  # full below max_seq_len: grow (never wrapped here)
            cap = min(2 * self._k.cap, self.max_seq_len)
            self._k.grow(cap, self._len)
            self._v.grow(cap, self._len)
        slot = (self._head + self._len) % self._k.cap
        self._k.put(slot, k_f, D)
        if self.asymmetric_v:
            v_min = v_f.min(dim=1, keepdim=True).values
            self._v.put(slot, v_f - v_min, D)
            self._v.zp[slot].copy_(v_min.squeeze(1))
        else:
            self._v.put(slot, v_f, D)
        self._len += 1

    def _order(self) -> torch.Tensor:
        return (torch.arange(self._len, device=self._k.packed.device) + self._head) % self._k.cap

    def get(self) -> Tuple[torch.Tensor, torch.Tensor]:
        """Full fp32 history: (K, V), both [B, H, T, D]."""
        if self._len == 0:
            raise RuntimeError("KV cache is empty")
        order = self._order()
        T, D = self._len, self.head_dim
        k_all = self._k.dequant(order)  # [BH, T, D]
        v_all = self._v.dequant(order)
        if self.asymmetric_v:
            zp = self._v.zp.index_select(0, order).t()  # [BH, T]
            v_all = v_all + zp.unsqueeze(-1)
        return (k_all.reshape(-1, self.n_heads, T, D), v_all.reshape(-1, self.n_heads, T, D))

    def get_quantized(self) -> Tuple[List[mx_tensor], List[mx_tensor]]:
        """Per-step packed slices (views of the ring), oldest first."""
        if self._len == 0:
            return [], []
        slots = self._order().tolist()
        return [self._k.step(s) for s in slots], [self._v.step(s) for s in slots]

    def reset(self) -> None:
        """Clear the cache between requests (the buffers are kept)."""
        self._head = 0
        self._len = 0

    @property
    def seq_len(self) -> int:
        return self._len

    def memory_bytes(self) -> int:
        """Bytes of the live steps: packed codes + scales of K and V, plus the
        V zero points (the reference's count)."""
        if self._len == 0:
            return 0
        step = self._k.row_bytes + self._k.rows * 4
        zp = self._k.rows * 4 if self.asymmetric_v else 0
        return self._len * (2 * step + zp)

    def compression_vs_fp16(self) -> float:
        T = self._len
        if T == 0:
            return 0.0
        fp16 = T * 2 * self.n_heads * self.head_dim * 2
        return fp16 / max(self.memory_bytes(), 1)

    def __repr__(self):
        return (f"kv_cache_quantizer(heads={self.n_heads}, dim={self.head_dim}, "
                f"dtype={self.dtype.name}, seq={self.seq_len}, "
                f"mem={self.memory_bytes() // 1024}KB)")
