"""save_quantized / load_quantized (mxtorch.py:9860-10004): the on-disk format.

tests/golden/ref_ckpt_int4d.pt was written by the reference's own
save_quantized (tests/golden/make_golden_dynamic.py).  Loading it here and
saving again must give the same dictionary: same keys, dtype names, packed
bytes, scales, shape, n and block."""
import os

import numpy as np
import pytest
import torch

import make_golden_dynamic as GD
import qtpytorch_b200 as mxb
from oracle import mx_oracle as O
from qtpytorch_b200.checkpoint import load_quantized, save_quantized

REF = os.path.join(os.path.dirname(__file__), "golden", "ref_ckpt_int4d.pt")


def _same_entry(a, b):
    assert a["dtype"] == b["dtype"] and list(a["shape"]) == list(b["shape"])
    assert int(a["n"]) == int(b["n"]) and int(a["block"]) == int(b["block"])
    assert torch.equal(a["packed"], b["packed"]) and a["packed"].dtype == b["packed"].dtype
    assert np.array_equal(a["scales"].numpy().view(np.uint32), b["scales"].numpy().view(np.uint32))


def test_reference_checkpoint_round_trip(tmp_path):
    ref = torch.load(REF, weights_only=True)
    m = load_quantized(REF, GD.make_ckpt_model)
    for key, e in ref.items():
        if key == "__mx_version__":
            continue
        mod, attr = key.rsplit(".", 1)
        t = getattr(dict(m.named_modules())[mod], attr)
        assert isinstance(t, mxb.mx_tensor) and t._mx_dtype.name == e["dtype"]
    out = tmp_path / "ours.pt"
    save_quantized(m, str(out))
    ours = torch.load(str(out), weights_only=True)
    assert ours.keys() == ref.keys() and ours["__mx_version__"] == 2
    for key in ref:
        if key != "__mx_version__":
            _same_entry(ours[key], ref[key])


def test_mx_linear_buffers_round_trip(tmp_path):
    # mx_linear's packed W^T, built from oracle codes (no GPU needed)
    w = torch.randn(64, 32, generator=torch.Generator().manual_seed(5))
    p, s, n = O.quantize(w.t().contiguous().numpy(), 4, "int", 32)
    lin = mxb.mx_linear(64, 32, bias=False, mx_dtype="int4d", block=32)
    lin._mx_weight = mxb.mx_tensor(torch.from_numpy(p), torch.from_numpy(s), "int4d",
                                   (64, 32), n, 32)
    model = torch.nn.Sequential(lin)
    path = tmp_path / "lin.pt"
    save_quantized(model, str(path), include_mx_linear=True)
    saved = torch.load(str(path), weights_only=True)
    assert set(saved) == {"__mx_version__", "0._mx_weight"}
    back = load_quantized(str(path), lambda: torch.nn.Sequential(
        mxb.mx_linear(64, 32, bias=False, mx_dtype="int4d", block=32)))
    assert torch.equal(back[0]._mx_weight._mx_packed, lin._mx_weight._mx_packed)
    # the reference format alone skips mx_linear modules, as the reference does
    save_quantized(model, str(path))
    assert set(torch.load(str(path), weights_only=True)) == {"__mx_version__"}


@pytest.mark.gpu
def test_load_state_dict_quantizes_on_gpu(tmp_path):
    sd_path = tmp_path / "sd.pt"
    ref_model = GD.make_ckpt_model()
    torch.save(ref_model.state_dict(), str(sd_path))
    m = load_quantized(str(sd_path), GD.make_ckpt_model, {r"^0$": "int4d", r"^2$": "float32"},
                       32, device="cuda")
    w = m[0].weight
    assert isinstance(w, mxb.mx_tensor) and w._mx_packed.is_cuda
    p, s, _ = O.quantize(ref_model[0].weight.detach().numpy(), 4, "int", 32)
    assert np.array_equal(w._mx_packed.cpu().numpy(), p)
    assert np.array_equal(w._mx_scales.cpu().numpy().view(np.uint32), s.view(np.uint32))
    assert isinstance(m[2].weight, torch.nn.Parameter) and m[2].weight.is_cuda
    x = torch.randn(3, 64, device="cuda")
    y = m(x)
    w_dq = torch.from_numpy(O.dequantize(p, s, 4, "int", (32, 64), 32)).cuda()
    b_dq = m[0].bias.dequantize()
    h = torch.relu(x @ w_dq.t() + b_dq)
    ref = h @ ref_model[2].weight.detach().cuda().t() + ref_model[2].bias.detach().cuda()
    assert torch.allclose(y, ref, rtol=1e-5, atol=1e-5)
