"""On-disk format: ``save_quantized`` / ``load_quantized`` (mxtorch.py:9860-10004).

The file is the reference's: ``torch.save`` of a dict with
``"__mx_version__": 2`` and, per quantized attribute, ``"<module>.<attr>" ->
{"dtype": name, "packed": int8 CPU tensor, "scales": fp32 CPU tensor,
"shape": list, "n": int, "block": int}``.  Files written here load in the
reference and the reference's files load here.  Reading uses
``torch.load(weights_only=True)``: the format holds only tensors, strings,
lists and ints, so no pickled code is executed.

A loaded attribute replaces the module's parameter with an mx_tensor
buffer; torch ops on it (``F.linear`` in ``nn.Linear.forward``) dequantize
it through the CUDA kernel.
"""
from __future__ import annotations

import re
from typing import Callable, Dict, Optional, Union

import torch
import torch.nn as nn

from . import _lib as L
from .dtypes import get_mx_dtype
from .linear import mx_linear
from .tensor import mx_tensor

MX_VERSION = 2
_FLOAT_NAMES = ("float32", "fp32", "float", "float16", "bfloat16")


def _payload(p) -> Optional[mx_tensor]:
    if isinstance(p, mx_tensor):
        return p
    if isinstance(p, nn.Parameter) and isinstance(p.data, mx_tensor):
        return p.data
    inner = getattr(p, "_mx_payload", None)
    return inner if isinstance(inner, mx_tensor) else None


def _entry(t: mx_tensor) -> dict:
    return {"dtype": t._mx_dtype.name, "packed": t._mx_packed.cpu(),
            "scales": t._mx_scales.cpu(), "shape": list(t._mx_orig_shape), "n": t._mx_n,
            "block": t._mx_block}


def save_quantized(model: nn.Module, path: str, include_mx_linear: bool = False) -> str:
    """Write the packed codes + scales of every ``weight`` / ``bias`` that is
    an mx_tensor (mxtorch.py:9860-9898).  ``include_mx_linear`` also writes
    ``mx_linear`` modules' packed buffers as ``<module>._mx_weight`` /
    ``._mx_bias`` (the reference's writer skips its own mx_linear modules;
    ``load_quantized`` here restores those keys, the reference's reader does
    not know them)."""
    ckpt: Dict[str, object] = {"__mx_version__": MX_VERSION}
    for name, module in model.named_modules():
        for attr in ("weight", "bias"):
            t = _payload(module._buffers.get(attr, module._parameters.get(attr)))
            if t is None and not isinstance(module, mx_linear):
                t = _payload(getattr(module, attr, None))
            if t is not None:
                ckpt[f"{name}.{attr}"] = _entry(t)
        if include_mx_linear and isinstance(module, mx_linear):
            for attr in ("_mx_weight", "_mx_bias"):
                t = module._buffers.get(attr)
                if isinstance(t, mx_tensor):
                    ckpt[f"{name}.{attr}"] = _entry(t)
    torch.save(ckpt, path)
    return path


def _set_mx(mod: nn.Module, attr: str, t: mx_tensor) -> None:
    if attr in mod._parameters:
        del mod._parameters[attr]
    if attr in mod._buffers or not hasattr(mod, attr):
        mod._buffers[attr] = t
    else:
        setattr(mod, attr, t)


def load_quantized(checkpoint_path: str, model_class: Callable[..., nn.Module],
                   dtype: Union[str, Dict[str, str]] = "int4d", block_size: int = 128,
                   model_kwargs: Optional[Dict] = None, device: str = "cpu") -> nn.Module:
    """Build ``model_class(**model_kwargs)`` and fill it from a checkpoint
    (mxtorch.py:9901-10004): an MX-native file restores the packed tensors as
    written; a plain state dict is quantized tensor by tensor with the dtype
    whose regex (``dtype`` dict, or one name for all) first matches the
    module name, on the CUDA kernels (the packed result then moves to
    ``device``); float dtype names and unmatched modules keep fp32 copies."""
    model = model_class(**(model_kwargs or {}))
    ckpt = torch.load(checkpoint_path, map_location="cpu", weights_only=True)
    modules = dict(model.named_modules())
    if isinstance(ckpt, dict) and "__mx_version__" in ckpt:
        for key, entry in ckpt.items():
            if key == "__mx_version__":
                continue
            parts = key.rsplit(".", 1)
            if len(parts) != 2 or parts[0] not in modules:
                continue
            t = mx_tensor(entry["packed"].to(device), entry["scales"].to(device),
                          get_mx_dtype(entry["dtype"]), torch.Size(entry["shape"]),
                          int(entry["n"]), int(entry["block"]))
            _set_mx(modules[parts[0]], parts[1], t)
        return model
    state = ckpt.get("state_dict") or ckpt.get("model") or ckpt if isinstance(ckpt, dict) else ckpt
    if not isinstance(state, dict):
        raise ValueError(f"Cannot parse checkpoint at {checkpoint_path}")
    dmap = {".*": dtype} if isinstance(dtype, str) else dtype
    by_module: Dict[str, Dict[str, torch.Tensor]] = {}
    for key, tensor in state.items():
        if not isinstance(tensor, torch.Tensor):
            continue
        parts = key.rsplit(".", 1)
        mod_n, attr_n = (parts[0], parts[1]) if len(parts) == 2 else ("", parts[0])
        by_module.setdefault(mod_n, {})[attr_n] = tensor
    qdev = torch.device(device) if torch.device(device).type == "cuda" else torch.device("cuda")
    for mod_name, attrs in by_module.items():
        target = next((dt for pat, dt in dmap.items() if re.search(pat, mod_name)), None)
        mod = modules.get(mod_name)
        if mod is None:
            continue
        for attr_n, tensor in attrs.items():
            p = getattr(mod, attr_n, None)
            if p is None:
                continue
            if target and target not in _FLOAT_NAMES:
                if not torch.cuda.is_available():
                    raise L.MxbError("load_quantized: quantizing a state dict needs a CUDA "
                                     "device (the mxb kernels run on CUDA only)")
                t = mx_tensor.quantize(tensor.float().to(qdev), get_mx_dtype(target), block_size)
                _set_mx(mod, attr_n, t._moved(torch.device(device)))
            elif isinstance(p, nn.Parameter):
                with torch.no_grad():
                    p.data.copy_(tensor)
    for name, mod in modules.items():
        for pname, prm in list(mod._parameters.items()):
            if prm is not None and prm.device != torch.device(device):
                mod._parameters[pname] = nn.Parameter(prm.data.to(device), prm.requires_grad)
    return model
