"""Random sign vectors for the Hadamard (``h``) variants.

The sign vector is drawn exactly as the reference's ``hadamard_rotation``
(mxtorch.py:2859-2864): ``randint(0, 2, (dim,))*2 - 1`` from a torch CPU
generator seeded with the dtype's seed, ``dim`` = next power of two of the
rotated length.  It is generated on the host once per (length, seed) and
cached on each device; the rotation itself runs in the CUDA library.
"""
from __future__ import annotations

import math
from typing import Dict, Tuple

import torch

_CACHE: Dict[Tuple[int, int, str], torch.Tensor] = {}


def pow2ceil(d: int) -> int:
    return 1 << math.ceil(math.log2(max(d, 1)))


def sign_vector(d: int, seed: int) -> torch.Tensor:
    """fp32 ±1 vector of length pow2ceil(d) on the CPU."""
    n = pow2ceil(d)
    gen = torch.Generator()
    gen.manual_seed(seed)
    return torch.randint(0, 2, (n,), generator=gen).float() * 2 - 1


def device_signs(d: int, seed: int, device) -> torch.Tensor:
    """The sign vector resident on ``device`` (cached)."""
    key = (d, seed, str(device))
    t = _CACHE.get(key)
    if t is None:
        t = sign_vector(d, seed).to(device)
        _CACHE[key] = t
    return t
