"""Generate golden vectors by running the reference mxtorch CPU path.

Run in a container that has the reference checked out (it is not needed at
test time; the fixtures are committed):

    PYTHONHASHSEED=0 PYTHONDONTWRITEBYTECODE=1 \
        python tests/golden/make_golden.py /path/to/qtpytorch

PYTHONHASHSEED=0 pins the reference's Hadamard seed (``hash(dt.name)``).
Inputs are drawn from torch's CPU generator with the seeds recorded in
``cases.py`` so the tests can regenerate them instead of storing them.
Outputs go to ``tests/golden/golden.npz``.
"""
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import cases  # noqa: E402


def main(ref_dir: str) -> None:
    if os.environ.get("PYTHONHASHSEED") != "0":
        raise SystemExit("run with PYTHONHASHSEED=0")
    sys.path.insert(0, ref_dir)
    import mxtorch as mx  # the reference

    torch.set_num_threads(1)
    out = {}

    def put(key, t):
        # large dequantized outputs are functions of packed+scales; skip them
        if key.endswith(("/dequant", "/dequant_ref_literal", "/rotated")) and key.split("/")[0] in cases.BIG_KEYS:
            return
        if isinstance(t, torch.Tensor):
            t = t.detach().cpu().numpy()
        out[key] = np.asarray(t)

    # known-answer packing test (mxtorch_test.py:86-93)
    vals = torch.tensor([3, -2, 7, -8, 0, 1, -1, 4], dtype=torch.int8)
    put("kat_pack4", mx.bit_packer.pack(vals, 4))
    put("kat_pack2", mx.bit_packer.pack(torch.tensor([1, -2, 0, -1, 1, -2, 0, 1], dtype=torch.int8), 2))
    put("kat_pack1", mx.bit_packer.pack(torch.tensor([0, 1, 0, 1, 1, 0, 1, 0], dtype=torch.int8), 1))

    # quantize / dequantize cases
    for c in cases.QUANT_CASES:
        x = cases.make_input(c)
        dt = mx.get_mx_dtype(c["dtype"])
        q = mx.mx_tensor.quantize(x, dt, c["block"])
        key = c["key"]
        put(f"{key}/packed", q._mx_packed)
        put(f"{key}/scales", q._mx_scales)
        put(f"{key}/n", np.int64(q._mx_n))
        if dt.is_hadamard:
            d = x.shape[-1] if x.ndim >= 2 else x.numel()
            n2 = 1 << int(np.ceil(np.log2(max(d, 1))))
            rot = mx.hadamard_rotation(n2, seed=hash(dt.name) % (2 ** 31))
            put(f"{key}/signs", rot.signs)
            put(f"{key}/seed", np.int64(hash(dt.name) % (2 ** 31)))
            xr = x.float() if x.ndim >= 2 else x.float().reshape(1, -1)
            put(f"{key}/rotated", rot.rotate(xr))
            # contract for h dequantize: inverse rotation along the last dim
            flat = mx._dequant(q._mx_packed, q._mx_scales, dt.base, q._mx_n, c["block"])
            put(f"{key}/dequant", rot.unrotate(flat.reshape(xr.shape)).reshape(x.shape))
            put(f"{key}/dequant_ref_literal", q.dequantize())
        else:
            put(f"{key}/dequant", q.dequantize())

    # config 1 GEMM: A 64x128 @ B 128x64 int8d (and other widths)
    for c in cases.GEMM_CASES:
        a, b = cases.make_gemm_inputs(c)
        dt = mx.get_mx_dtype(c["dtype"])
        qa = mx.mx_tensor.quantize(a, dt, c["block"])
        qb = mx.mx_tensor.quantize(b, mx.get_mx_dtype(c.get("dtype_b", c["dtype"])), c["block"])
        qc = qa @ qb
        key = c["key"]
        put(f"{key}/c_packed", qc._mx_packed)
        put(f"{key}/c_scales", qc._mx_scales)
        put(f"{key}/c_bits", np.int64(qc._mx_dtype.bits))
        put(f"{key}/c_block", np.int64(qc._mx_block))
        put(f"{key}/c_dtype", np.array(qc._mx_dtype.name))
        put(f"{key}/c_dequant", qc.dequantize())

    # weight-only linear (mx_linear.from_linear + forward, bias-free)
    for c in cases.LINEAR_CASES:
        lin, x = cases.make_linear_inputs(c)
        ml = mx.mx_linear.from_linear(lin, mx.get_mx_dtype(c["dtype"]), c["block"])
        w = ml._mx_weight
        key = c["key"]
        put(f"{key}/w_packed", w._mx_packed)
        put(f"{key}/w_scales", w._mx_scales)
        with torch.no_grad():
            put(f"{key}/y", ml(x))

    # raw WHT
    g = torch.Generator().manual_seed(11)
    xw = torch.randn(2, 1024, generator=g)
    put("wht/y", mx._fast_hadamard_transform(xw))

    np.savez_compressed(os.path.join(HERE, "golden.npz"), **out)
    print("wrote", len(out), "arrays")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "../reference")
