"""ctypes binding of the mxb C ABI (include/mxb.h).

The shared library is built in-tree (``python -m qtpytorch_b200.build``) and
loaded from this package's directory.  There is no fallback: if the library
is missing or a call fails, an exception says why.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libmxb.so")

MXB_OK = 0
ERRORS = {
    -1: "MXB_E_SHAPE (unsupported or inconsistent sizes)",
    -2: "MXB_E_DTYPE (unsupported bits / kind / variant)",
    -3: "MXB_E_ALIGN (pointer alignment)",
    -4: "MXB_E_CUDA (CUDA runtime error)",
    -6: "MXB_E_ARG (null pointer or invalid argument)",
    -7: "MXB_E_WORKSPACE (workspace missing or too small)",
}
F32, BF16 = 0, 1
KIND_INT, KIND_FLOAT = 0, 1
VAR_BASE, VAR_H = 0, 1
MODE_PARITY, MODE_FAST = 0, 1

_i64, _int, _sz, _vp = C.c_int64, C.c_int, C.c_size_t, C.c_void_p

# name -> (restype, argtypes); the single source for the exported symbol list
PROTOTYPES = {
    "mxb_version": (_int, []),
    "mxb_last_error": (C.c_char_p, []),
    "mxb_launch_count": (C.c_uint64, []),
    "mxb_device_error": (_int, [_int]),
    "mxb_linear_wonly_noalloc": (_int, [_vp, _int, _i64, _i64, _vp, _vp, _i64, _int, _int, _int,
                                        _vp, _vp]),
    "mxb_packed_bytes": (_sz, [_i64, _int, _int]),
    "mxb_quantize_workspace_size": (_sz, [_i64, _i64, _int, _int, _int, _int]),
    "mxb_quantize": (_int, [_vp, _int, _i64, _i64, _int, _int, _int, _int, _vp, _vp, _vp,
                            _vp, _sz, _vp]),
    "mxb_dynamic_quantize_workspace_size": (_sz, [_i64, _i64]),
    "mxb_dynamic_quantize": (_int, [_vp, _int, _i64, _i64, _int, _vp, _vp, _vp, _sz, _vp]),
    "mxb_dequantize": (_int, [_vp, _vp, _i64, _i64, _int, _int, _int, _int, _vp, _vp, _vp]),
    "mxb_dequantize_relu": (_int, [_vp, _vp, _i64, _int, _int, _int, _vp, _vp]),
    "mxb_dequantize_silu_mul": (_int, [_vp, _vp, _vp, _vp, _i64, _int, _int, _int, _vp, _vp]),
    "mxb_hadamard_rows": (_int, [_vp, _i64, _i64, _vp, _int, _vp, _vp]),
    "mxb_qgemm_workspace_size": (_sz, [_i64, _i64, _i64, _int, _int]),
    "mxb_qgemm": (_int, [_vp, _vp, _i64, _vp, _vp, _i64, _i64, _i64, _i64, _int, _int, _int,
                         _vp, _vp, _vp, _vp, _sz, _vp]),
    "mxb_qgemm_kmajor_workspace_size": (_sz, [_i64, _i64, _i64, _int, _int]),
    "mxb_qgemm_kmajor": (_int, [_vp, _vp, _i64, _vp, _vp, _i64, _i64, _i64, _i64, _int, _int,
                                _int, _vp, _vp, _vp, _vp, _sz, _vp]),
    "mxb_qgemm_sharded": (_int, [_vp, _vp, _i64, _vp, _vp, _i64, _i64, _i64, _i64, _int, _int,
                                 _i64, _i64, _int, _vp, _vp, _vp, _sz, _vp]),
    "mxb_qgemm_sharded_sync": (_int, [_vp, _vp, _i64, _vp, _vp, _i64, _i64, _i64, _i64, _int,
                                      _int, _i64, _i64, _int, _int, _vp, _vp, _vp, _vp, _sz,
                                      _vp]),
    "mxb_peer_barrier": (_int, [_int, _int, _vp, _vp]),
    "mxb_allgather_cols": (_int, [_int, _int, _i64, _i64, _vp, _vp, _vp, _vp, _vp]),
    "mxb_ipc_open": (_int, [_vp, _i64, _vp]),
    "mxb_ipc_close": (_int, [_vp]),
    "mxb_linear_wonly_workspace_size": (_sz, [_i64, _i64, _i64, _int, _int, _int, _int]),
    "mxb_linear_wonly": (_int, [_vp, _int, _i64, _i64, _vp, _vp, _i64, _int, _int, _int, _int,
                                _vp, _vp, _sz, _vp]),
    "mxb_hadamard_cross": (_int, [_vp, _i64, _i64, _int, _vp, _vp, _vp]),
    "mxb_linear_wonly_kmajor": (_int, [_vp, _int, _i64, _i64, _vp, _vp, _i64, _int, _int, _int,
                                       _int, _vp, _vp]),
}

_lib = None
_lock = threading.Lock()


class MxbError(RuntimeError):
    pass


def load():
    """Load libmxb.so (once) and bind its prototypes."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise MxbError(
                    f"{LIB_PATH} is missing: build it with `python -m qtpytorch_b200.build`")
            lib = C.CDLL(LIB_PATH)
            for name, (res, args) in PROTOTYPES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def check(rc: int, what: str) -> None:
    if rc != MXB_OK:
        msg = ERRORS.get(rc, f"status {rc}")
        detail = load().mxb_last_error().decode(errors="replace")
        raise MxbError(f"{what} failed: {msg}" + (f" [{detail}]" if detail else ""))


def ptr(t) -> int:
    return 0 if t is None else t.data_ptr()


def stream_of(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(t: torch.Tensor, what: str) -> None:
    if not t.is_cuda:
        raise MxbError(f"{what}: tensor is on {t.device}; the mxb kernels run on CUDA only")


def workspace(nbytes: int, device) -> torch.Tensor | None:
    if nbytes <= 0:
        return None
    return torch.empty(nbytes, dtype=torch.uint8, device=device)
