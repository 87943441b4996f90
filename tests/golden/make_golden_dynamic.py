"""Golden vectors for the dynamic-quantize / full-int8 linear path, made by
running the reference mxtorch CPU path (not needed at test time).

    PYTHONHASHSEED=0 PYTHONDONTWRITEBYTECODE=1 \
        python tests/golden/make_golden_dynamic.py /path/to/qtpytorch

Covers ``dynamic_quantize`` (mxtorch.py:2665-2712, every granularity),
``fused_int8_linear`` (3910-3960, CPU branch: dequantize + F.linear),
``mx_dynamic_linear`` (8870-8978), ``fused_linear_relu`` (4012-4074, CPU
branch), ``fused_silu_and_mul`` (4077-4109, CPU branch) and
``kv_cache_quantizer`` (2998-3119); ``save_quantized`` (9860-9898) of a
model loaded by ``load_quantized`` (9901-10004) from a plain state dict,
written to ``ref_ckpt_int4d.pt`` (the reference's on-disk format).  Inputs come from torch's CPU generator
with the seeds in the ``*_CASES`` lists so the
tests regenerate them.  Output: ``tests/golden/golden_dynamic.npz``.
"""
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

# key, dtype, granularity, shape, seed, input dtype, block (per_block only)
DYN_CASES = [
    ("tok_int8d", "int8d", "per_token", (16, 256), 101, "fp32", 64),
    ("tok_int4d", "int4d", "per_token", (8, 384), 102, "fp32", 64),
    ("tok_int2d", "int2d", "per_token", (8, 130), 103, "fp32", 64),
    ("tok_int8d_bf16", "int8d", "per_token", (4, 512), 104, "bf16", 64),
    ("tok_int8d_3d", "int8d", "per_token", (2, 3, 96), 105, "fp32", 64),
    ("tensor_int8d", "int8d", "per_tensor", (1000,), 106, "fp32", 64),
    ("tensor_int4d", "int4d", "per_tensor", (7, 33), 107, "fp32", 64),
    ("block_int8d", "int8d", "per_block", (4, 256), 108, "fp32", 64),
    ("chan_int8d", "int8d", "per_channel", (64, 32), 109, "fp32", 64),
]

# key, M, K, N, x granularity, weight block, bias, seed
FUSED_CASES = [
    ("f_tok_b128", 8, 256, 96, "per_token", 128, True, 201),
    ("f_tok_nobias", 5, 384, 64, "per_token", 128, False, 202),
    ("f_block128", 16, 256, 128, "per_block128", 128, True, 203),
    ("f_tc", 256, 512, 256, "per_token", 128, True, 204),
]

# key, tokens, in, out, weight dtype, bias, seed
DLIN_CASES = [
    ("dl_int4d", 6, 256, 96, "int4d", True, 301),
    ("dl_int8d_nobias", 3, 128, 64, "int8d", False, 302),
]

# key, M, K, N, dtype, bias, weight given as mx_tensor [in, out], seed
RELU_CASES = [
    ("r_int8d", 8, 256, 96, "int8d", True, False, 401),
    ("r_int4d_mx", 5, 256, 128, "int4d", False, True, 402),
    ("r_int8d_3d", 6, 128, 64, "int8d", True, False, 403),
]

# key, dtype, shape, block, seed
SILU_CASES = [
    ("s_int8d", "int8d", (8, 1000), 128, 501),
    ("s_int4d", "int4d", (4, 4096), 128, 502),
    ("s_float4d", "float4d", (3, 512), 32, 503),
    ("s_int2d_b8", "int2d", (2, 96), 8, 504),
]

# key, B, H, D, dtype, max_seq_len, steps, asymmetric_v, layout, seed
KV_CASES = [
    ("kv_int8d", 2, 4, 64, "int8d", 16, 7, True, "bhtd", 601),
    ("kv_int4d_evict", 1, 3, 128, "int4d", 5, 12, True, "bhtd", 602),
    ("kv_int8d_sym", 2, 2, 32, "int8d", 70, 67, False, "bthd", 603),
    ("kv_int4dh", 1, 2, 64, "int4dh", 8, 9, True, "bhtd", 604),
]


def make_kv_steps(c):
    _, B, H, D, _, _, steps, _, layout, seed = c
    g = torch.Generator().manual_seed(seed)
    shape = (B, H, 1, D) if layout == "bhtd" else (B, 1, H, D)
    return [(torch.randn(*shape, generator=g), torch.randn(*shape, generator=g) + 0.5)
            for _ in range(steps)]


def make_ckpt_model():
    """The model class of the checkpoint fixture: Linear(64, 32), ReLU,
    Linear(32, 16), weights from a fixed seed."""
    torch.manual_seed(701)
    return torch.nn.Sequential(torch.nn.Linear(64, 32), torch.nn.ReLU(), torch.nn.Linear(32, 16))


def make_relu_inputs(c):
    key, M, K, N, _, has_bias, _, seed = c
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g)
    if key.endswith("_3d"):
        x = x.view(2, M // 2, K)
    w = torch.randn(N, K, generator=g) * 0.05
    b = torch.randn(N, generator=g) if has_bias else None
    return x, w, b


def make_silu_inputs(c):
    _, _, shape, _, seed = c
    g = torch.Generator().manual_seed(seed)
    return torch.randn(*shape, generator=g) * 3, torch.randn(*shape, generator=g)


def make_dyn_input(c):
    _, _, _, shape, seed, in_dt, _ = c
    x = torch.randn(*shape, generator=torch.Generator().manual_seed(seed)) * 2.0
    return x.bfloat16() if in_dt == "bf16" else x


def make_fused_inputs(c):
    _, M, K, N, _, _, has_bias, seed = c
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g)
    w = torch.randn(N, K, generator=g) * 0.05
    b = torch.randn(N, generator=g) if has_bias else None
    return x, w, b


def make_dlin_inputs(c):
    _, T, K, N, _, has_bias, seed = c
    g = torch.Generator().manual_seed(seed)
    lin = torch.nn.Linear(K, N, bias=has_bias)
    with torch.no_grad():
        lin.weight.copy_(torch.randn(N, K, generator=g) * 0.05)
        if has_bias:
            lin.bias.copy_(torch.randn(N, generator=g))
    x = torch.randn(T, K, generator=g)
    return lin, x


def main(ref_dir: str) -> None:
    if os.environ.get("PYTHONHASHSEED") != "0":
        raise SystemExit("run with PYTHONHASHSEED=0")
    sys.path.insert(0, ref_dir)
    import mxtorch as mx  # the reference

    torch.set_num_threads(1)
    out = {}
    for c in DYN_CASES:
        key, dt, gran, _, _, _, block = c
        q = mx.dynamic_quantize(make_dyn_input(c), dt, gran, block)
        out[f"{key}/packed"] = q._mx_packed.numpy()
        out[f"{key}/scales"] = q._mx_scales.numpy()
        out[f"{key}/block"] = np.int64(q._mx_block)
        out[f"{key}/n"] = np.int64(q._mx_n)
        out[f"{key}/dequant"] = q.dequantize().float().numpy()
    for c in FUSED_CASES:
        key, M, K, N, gran, wblock, _, _ = c
        x, w, b = make_fused_inputs(c)
        if gran == "per_token":
            xq = mx.dynamic_quantize(x, "int8d", "per_token")
        else:
            xq = mx.mx_tensor.quantize(x, mx.get_mx_dtype("int8d"), 128)
        wq = mx.mx_tensor.quantize(w, mx.get_mx_dtype("int8d"), wblock)
        y = mx.fused_int8_linear(xq, wq, b, wblock)
        out[f"{key}/out"] = y.numpy()
    for c in DLIN_CASES:
        key, _, _, _, wdt, _, _ = c
        lin, x = make_dlin_inputs(c)
        m = mx.mx_dynamic_linear.from_linear(lin, wdt, "int8d")
        out[f"{key}/out"] = m(x).detach().numpy()
        out[f"{key}/w_packed"] = m.weight._mx_packed.numpy()
        out[f"{key}/w_scales"] = m.weight._mx_scales.numpy()
    for c in RELU_CASES:
        key, _, _, _, dt, _, w_mx, _ = c
        x, w, b = make_relu_inputs(c)
        mdt = mx.get_mx_dtype(dt)
        if w_mx:
            y = mx.fused_linear_relu(x, mx.mx_tensor.quantize(w.t(), mdt, 128), b, 128)
        else:
            y = mx.fused_linear_relu(x, w, b, 128, mdt)
        out[f"{key}/out"] = y.numpy()
    for c in SILU_CASES:
        key, dt, _, block, _ = c
        g, u = make_silu_inputs(c)
        mdt = mx.get_mx_dtype(dt)
        y = mx.fused_silu_and_mul(mx.mx_tensor.quantize(g, mdt, block),
                                  mx.mx_tensor.quantize(u, mdt, block))
        out[f"{key}/out"] = y.numpy()
    for c in KV_CASES:
        key, _, H, D, dt, max_len, _, asym, _, _ = c
        cache = mx.kv_cache_quantizer(H, D, dt, max_seq_len=max_len, asymmetric_v=asym)
        for k, v in make_kv_steps(c):
            cache.append_kv(k, v)
        K, V = cache.get()
        out[f"{key}/k"] = K.numpy()
        out[f"{key}/v"] = V.numpy()
        out[f"{key}/seq_len"] = np.int64(cache.seq_len)
        out[f"{key}/memory_bytes"] = np.int64(cache.memory_bytes())
    import tempfile
    with tempfile.TemporaryDirectory() as td:
        sd_path = os.path.join(td, "sd.pt")
        torch.save(make_ckpt_model().state_dict(), sd_path)
        m = mx.load_quantized(sd_path, make_ckpt_model, "int4d", 32)
        mx.save_quantized(m, os.path.join(HERE, "ref_ckpt_int4d.pt"))
    np.savez_compressed(os.path.join(HERE, "golden_dynamic.npz"), **out)
    print(f"wrote {len(out)} arrays")


if __name__ == "__main__":
    main(sys.argv[1])
