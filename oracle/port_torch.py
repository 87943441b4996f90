"""The configs[1] job (int8d quantize of A and B, packed int matmul, int16d
requantize) on the host cores with torch CPU ops: the CPU baseline that
bench.py times on the GPU box, where the reference itself cannot run.

TEST / BASELINE INFRASTRUCTURE ONLY: imported by bench.py's CPU-baseline and
reference legs and by tests/, never by the product package.

It is the numpy oracle's algorithm (oracle/mx_oracle.py, whose results it
reproduces bit for bit: tests/test_oracle_golden.py) written with the same
multithreaded torch CPU kernels the reference's CPU path runs
(mxtorch.py:1426-1463 `_quant_int`, 1299-1385 `_qscale_matmul`, 870-985
`bit_packer`), so its time stands in for the reference's on the same host:
oracle/calibrate_port.py records the ratio of the two in this container.
"""
from __future__ import annotations

import math

import torch


def quantize_int(x: torch.Tensor, bits: int, block: int):
    """(codes int32 [nb*block], scales fp32 [nb], n): per block
    si = max_int / max(amax, 1e-12) (reciprocal then multiply, as torch's
    scalar division), scale = 1/si, code = round(clamp(x*si))."""
    flat = x.float().reshape(-1)
    n = flat.numel()
    nb = math.ceil(n / block)
    if nb * block != n:
        flat = torch.cat([flat, flat.new_zeros(nb * block - n)])
    blk = flat.reshape(nb, block)
    max_int = float((1 << (bits - 1)) - 1)
    si = max_int / blk.abs().amax(dim=1).clamp(min=1e-12)
    scales = si.reciprocal()
    codes = (blk * si.unsqueeze(1)).clamp(-max_int, max_int).round_().to(torch.int32)
    return codes.reshape(-1), scales, n


def qscale_matmul(a_codes, a_scales, b_codes, b_scales, M, K, N, block, out_bits):
    """C = sum_kb fl(fl(P_kb * sa[:, kb]) * sb[kb, :]) in kb order (B's scales
    viewed [K/block, N]), P_kb the exact integer product in fp32; then the
    requantize over flat blocks.  Returns (codes int32 [M*N], scales)."""
    A = a_codes.reshape(M, K).float()
    B = b_codes.reshape(K, N).float()
    kb_n = math.ceil(K / block)
    sa = (a_scales.reshape(M, kb_n) if a_scales.numel() == M * kb_n
          else a_scales.new_ones(M, kb_n))
    sb = (b_scales.reshape(kb_n, N) if b_scales.numel() == kb_n * N
          else b_scales.new_ones(kb_n, N))
    C = torch.zeros(M, N, dtype=torch.float32)
    for kb in range(kb_n):
        k0, k1 = kb * block, min(kb * block + block, K)
        P = torch.mm(A[:, k0:k1], B[k0:k1, :])
        C += P * sa[:, kb:kb + 1] * sb[kb:kb + 1, :]
    max_out = float((1 << (out_bits - 1)) - 1)
    flat = C.reshape(-1)
    nb = math.ceil(flat.numel() / block)
    if nb * block != flat.numel():
        flat = torch.cat([flat, flat.new_zeros(nb * block - flat.numel())])
    blk = flat.reshape(nb, block)
    cs = blk.abs().amax(dim=1).clamp(min=1e-12) / max_out
    codes = (blk / cs.unsqueeze(1)).clamp(-max_out, max_out).round_().to(torch.int32)
    return codes.reshape(-1)[: M * N], cs


def pack16(codes: torch.Tensor) -> torch.Tensor:
    """Two 16-bit codes per int32 word, low half first."""
    c = codes.to(torch.int64)
    if c.numel() % 2:
        c = torch.cat([c, c.new_zeros(1)])
    return (((c[1::2] & 0xFFFF) << 16) | (c[0::2] & 0xFFFF)).to(torch.uint32).view(torch.int32)


def int8_job(a: torch.Tensor, b: torch.Tensor, block: int = 128):
    """quantize A and B to int8d, A @ B, requantize to int16d: the whole
    configs[1] job.  Returns (packed int32 words, scales)."""
    M, K = a.shape
    N = b.shape[1]
    ca, sa, _ = quantize_int(a, 8, block)
    cb, sb, _ = quantize_int(b, 8, block)
    codes, cs = qscale_matmul(ca, sa, cb, sb, M, K, N, block, 16)
    return pack16(codes), cs
