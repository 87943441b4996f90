"""MX dtype registry: names, bit widths, variants and representable ranges.

Mirrors the reference's dtype system (mxtorch.py:413-655): a dtype is the
tuple (kind, bits, mode, variant) and its name is ``f"{kind}{bits}{mode}{variant}"``
(``int4d``, ``float4d``, ``int4dh`` ...).  Only metadata lives here; the
arithmetic is in the CUDA library.

The Hadamard-variant seed follows mxtorch.py:1723 (``hash(dt.name) % 2**31``).
CPython salts ``str.__hash__`` per process, so the reference's rotation changes
from run to run unless ``PYTHONHASHSEED=0``.  This build pins the
``PYTHONHASHSEED=0`` value by computing CPython's SipHash-1-3 string hash with
the all-zero key, which makes packed ``h`` tensors reproducible across
processes and equal to the reference's output under ``PYTHONHASHSEED=0``.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass
from typing import Dict, Union

_VALID_BITS = (1, 2, 3, 4, 5, 6, 7, 8, 16, 32, 64, 128)
_VALID_MODES = ("d", "u")
_VALID_KINDS = ("int", "float")
_VALID_VARIANTS = ("", "h", "v", "s", "b", "2")

# Widths whose quantize / dequantize / matmul run on the CUDA library.
KERNEL_BITS = (1, 2, 4, 8)


@dataclass(frozen=True)
class mx_dtype:
    """One MX data type (mxtorch.py:428-547)."""

    kind: str
    bits: int
    mode: str
    variant: str = ""

    def __post_init__(self):
        if self.kind not in _VALID_KINDS:
            raise ValueError(f"Invalid kind {self.kind!r}")
        if self.bits not in _VALID_BITS:
            raise ValueError(f"Invalid bits {self.bits}")
        if self.mode not in _VALID_MODES:
            raise ValueError(f"Invalid mode {self.mode!r}")
        if self.variant not in _VALID_VARIANTS:
            raise ValueError(f"Invalid variant {self.variant!r}")

    @property
    def name(self) -> str:
        return f"{self.kind}{self.bits}{self.mode}{self.variant}"

    def __repr__(self):
        return f"mx.{self.name}"

    def __str__(self):
        return self.name

    is_float = property(lambda self: self.kind == "float")
    is_int = property(lambda self: self.kind == "int")
    is_down = property(lambda self: self.mode == "d")
    is_up = property(lambda self: self.mode == "u")
    is_bool = property(lambda self: self.variant == "b")
    is_stochastic = property(lambda self: self.variant == "s")
    is_hadamard = property(lambda self: self.variant == "h")
    is_vector = property(lambda self: self.variant == "v")
    is_base = property(lambda self: self.variant == "")
    is_double_prec = property(lambda self: self.variant == "2")

    @property
    def base(self) -> "mx_dtype":
        """The dtype with its variant suffix stripped (mxtorch.py:506-511)."""
        if self.variant == "":
            return self
        return _DTYPE_REGISTRY.get(f"{self.kind}{self.bits}{self.mode}", self)

    @property
    def max_val(self) -> float:
        """Largest code magnitude (mxtorch.py:514-526)."""
        if self.is_bool:
            return 1.0
        if self.is_int:
            if self.bits == 1:
                return 1.0
            return float((1 << (self.bits - 1)) - 1)
        fmax = {1: 1.0, 2: 1.5, 3: 3.5, 4: 6.0, 5: 14.0, 6: 28.0, 7: 56.0,
                8: 448.0, 16: 65504.0}
        return fmax.get(self.bits, float("inf"))

    @property
    def native_storage_bits(self) -> int:
        if self.bits <= 8:
            return 8
        if self.bits <= 16:
            return 16
        if self.bits <= 32:
            return 32
        return 64

    @property
    def pack_ratio(self) -> int:
        return self.native_storage_bits // self.bits

    @property
    def compression_vs_fp32(self) -> float:
        return 32.0 / self.bits

    @property
    def hadamard_seed(self) -> int:
        """Seed of the random sign vector for ``h`` dtypes (mxtorch.py:1723)."""
        return str_hash_seed0(self.name) % (2 ** 31)


_DTYPE_REGISTRY: Dict[str, mx_dtype] = {}
for _k in _VALID_KINDS:
    for _b in _VALID_BITS:
        for _m in _VALID_MODES:
            for _v in _VALID_VARIANTS:
                _dt = mx_dtype(_k, _b, _m, _v)
                _DTYPE_REGISTRY[_dt.name] = _dt


def get_mx_dtype(name: Union[str, mx_dtype]) -> mx_dtype:
    """Resolve a dtype name (mxtorch.py:560-583); raises ValueError if unknown."""
    if isinstance(name, mx_dtype):
        return name
    inner = getattr(name, "_mx", None)
    if isinstance(inner, mx_dtype):
        return inner
    if name not in _DTYPE_REGISTRY:
        raise ValueError(
            f"Unknown MX dtype {name!r}. Format: {{int|float}}{{bits}}{{d|u}}"
            f"[{{h|v|s|b}}]. Examples: int4d, float8u, int2dv, float4uh, int8us")
    return _DTYPE_REGISTRY[name]


def optimal_output_dtype(op: str, a: mx_dtype, b: mx_dtype) -> mx_dtype:
    """Output dtype of a quantized op (mxtorch.py:1393-1423).

    matmul: bits = min(32, a.bits + b.bits), snapped to the nearest valid
    width (ties to the wider one).
    """
    kind = "float" if (a.is_float or b.is_float) else "int"
    mode = "u" if (a.is_up or b.is_up) else "d"
    if op == "matmul":
        ideal = min(32, a.bits + b.bits)
    elif op in ("add", "sub"):
        ideal = min(a.bits, b.bits) + 1
    elif op == "mul":
        ideal = min(a.bits * 2, 32)
    else:
        ideal = max(a.bits, b.bits)
    best = min(_VALID_BITS, key=lambda x: (abs(x - ideal), -x))
    return get_mx_dtype(f"{kind}{best}{mode}")


# ── CPython str hash with PYTHONHASHSEED=0 ───────────────────────────────────
_M64 = (1 << 64) - 1


def _rotl(x: int, b: int) -> int:
    return ((x << b) | (x >> (64 - b))) & _M64


def _siphash13(data: bytes, k0: int = 0, k1: int = 0) -> int:
    """SipHash-1-3 (Aumasson & Bernstein), the string hash of CPython >= 3.11."""
    v0 = k0 ^ 0x736F6D6570736575
    v1 = k1 ^ 0x646F72616E646F6D
    v2 = k0 ^ 0x6C7967656E657261
    v3 = k1 ^ 0x7465646279746573

    def rnd(v0, v1, v2, v3):
        v0 = (v0 + v1) & _M64; v1 = _rotl(v1, 13); v1 ^= v0; v0 = _rotl(v0, 32)
        v2 = (v2 + v3) & _M64; v3 = _rotl(v3, 16); v3 ^= v2
        v0 = (v0 + v3) & _M64; v3 = _rotl(v3, 21); v3 ^= v0
        v2 = (v2 + v1) & _M64; v1 = _rotl(v1, 17); v1 ^= v2; v2 = _rotl(v2, 32)
        return v0, v1, v2, v3

    n = len(data)
    full = n // 8 * 8
    for i in range(0, full, 8):
        m = struct.unpack_from("<Q", data, i)[0]
        v3 ^= m
        v0, v1, v2, v3 = rnd(v0, v1, v2, v3)
        v0 ^= m
    tail = data[full:] + b"\0" * (7 - (n - full))
    last = ((n & 0xFF) << 56) | int.from_bytes(tail[:7], "little")
    v3 ^= last
    v0, v1, v2, v3 = rnd(v0, v1, v2, v3)
    v0 ^= last
    v2 ^= 0xFF
    for _ in range(3):
        v0, v1, v2, v3 = rnd(v0, v1, v2, v3)
    return v0 ^ v1 ^ v2 ^ v3


def str_hash_seed0(s: str) -> int:
    """``hash(s)`` as CPython computes it for an ASCII str under PYTHONHASHSEED=0."""
    data = s.encode("latin-1")
    if not data:
        return 0
    h = _siphash13(data)
    if h >= 1 << 63:
        h -= 1 << 64
    if h == -1:
        h = -2
    return h


# module-level aliases, as in the reference (mxtorch.py:606-655)
for _name, _dt in _DTYPE_REGISTRY.items():
    globals()[_name] = _dt
