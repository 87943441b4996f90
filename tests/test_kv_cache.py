"""kv_cache_quantizer (mxtorch.py:2998-3119) against fixtures made by running
the reference (tests/golden/make_golden_dynamic.py): append sequences with
eviction at max_seq_len, ring growth, symmetric and asymmetric V, both input
layouts.  get() is bit-exact.  For the `h` case the reference unrotates the
flattened step while this framework unrotates each head row, so that case is
checked against the oracle's row-wise restatement instead."""
import numpy as np
import pytest
import torch

import make_golden_dynamic as GD
import qtpytorch_b200 as mxb
from oracle import mx_oracle as O
from qtpytorch_b200 import _lib as L
from qtpytorch_b200.kv_cache import kv_cache_quantizer


def _u32(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def _is_h(c):
    return mxb.get_mx_dtype(c[4]).is_hadamard


def _oracle_kv(c):
    """The reference's list-of-steps cache restated with the oracle."""
    _, B, H, D, dt, max_len, _, asym, _, _ = c
    d = mxb.get_mx_dtype(dt)
    signs = mxb.sign_vector(D, d.hadamard_seed).numpy() if d.is_hadamard else None
    ks, vs = [], []
    for k, v in GD.make_kv_steps(c):
        kf = k.float().reshape(-1, D).numpy()
        vf = v.float().reshape(-1, D).numpy()
        if len(ks) >= max_len:
            ks.pop(0)
            vs.pop(0)
        kp, ksc, _ = O.quantize(kf, d.bits, d.kind, D, d.is_hadamard, signs)
        ks.append(O.dequantize(kp, ksc, d.bits, d.kind, kf.shape, D, d.is_hadamard, signs))
        if asym:
            vmin = vf.min(axis=1, keepdims=True)
            vsft = (vf - vmin).astype(np.float32)
            vp, vsc, _ = O.quantize(vsft, d.bits, d.kind, D, d.is_hadamard, signs)
            dq = O.dequantize(vp, vsc, d.bits, d.kind, vf.shape, D, d.is_hadamard, signs)
            vs.append((dq + vmin).astype(np.float32))
        else:
            vp, vsc, _ = O.quantize(vf, d.bits, d.kind, D, d.is_hadamard, signs)
            vs.append(O.dequantize(vp, vsc, d.bits, d.kind, vf.shape, D, d.is_hadamard, signs))
    T = len(ks)
    return (np.stack(ks, axis=1).reshape(-1, H, T, D), np.stack(vs, axis=1).reshape(-1, H, T, D))


@pytest.mark.parametrize("c", [c for c in GD.KV_CASES if not _is_h(c)], ids=lambda c: c[0])
def test_oracle_kv_cache_matches_reference(golden_dynamic, c):
    K, V = _oracle_kv(c)
    assert np.array_equal(_u32(K), _u32(golden_dynamic[f"{c[0]}/k"]))
    assert np.array_equal(_u32(V), _u32(golden_dynamic[f"{c[0]}/v"]))


def test_kv_cache_rejects_host_tensors():
    cache = kv_cache_quantizer(2, 32)
    with pytest.raises(L.MxbError):
        cache.append_kv(torch.zeros(1, 2, 1, 32), torch.zeros(1, 2, 1, 32))


@pytest.mark.gpu
@pytest.mark.parametrize("c", GD.KV_CASES, ids=lambda c: c[0])
def test_kv_cache_bit_exact(golden_dynamic, c):
    key, B, H, D, dt, max_len, steps, asym, _, _ = c
    cache = mxb.kv_cache_quantizer(H, D, dt, max_seq_len=max_len, asymmetric_v=asym)
    for k, v in GD.make_kv_steps(c):
        cache.append_kv(k.cuda(), v.cuda())
    g = golden_dynamic
    assert cache.seq_len == int(g[f"{key}/seq_len"]) == min(steps, max_len)
    assert cache.memory_bytes() == int(g[f"{key}/memory_bytes"])
    K, V = cache.get()
    Ko, Vo = _oracle_kv(c)
    assert np.array_equal(_u32(K.cpu().numpy()), _u32(Ko))
    assert np.array_equal(_u32(V.cpu().numpy()), _u32(Vo))
    if not _is_h(c):
        assert np.array_equal(_u32(K.cpu().numpy()), _u32(g[f"{key}/k"]))
        assert np.array_equal(_u32(V.cpu().numpy()), _u32(g[f"{key}/v"]))
    kq, vq = cache.get_quantized()
    assert len(kq) == len(vq) == cache.seq_len
    last = kq[-1].dequantize().cpu().numpy().reshape(-1)
    assert np.array_equal(_u32(last), _u32(Ko[:, :, -1, :].reshape(-1)))
    cache.reset()
    assert cache.seq_len == 0 and cache.memory_bytes() == 0
    with pytest.raises(RuntimeError):
        cache.get()
