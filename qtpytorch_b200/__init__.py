"""qtpytorch_b200 — B200-native (sm_100a) MX quantize / pack / packed matmul.

The reference's hot-path API (DHDev0/qtpytorch ``mxtorch``) on CUDA kernels:
``mx_tensor.quantize`` / ``dequantize`` / ``@``, ``mx_linear``, ``to_mx``,
``mx_matmul``, ``get_mx_dtype``, ``register_kernel``, ``dynamic_quantize``,
``fused_int8_linear``, ``mx_dynamic_linear``, ``fused_linear_relu``,
``fused_silu_and_mul``, ``kv_cache_quantizer``, ``save_quantized``, ``load_quantized``.
"""
from .dtypes import (  # noqa: F401
    _DTYPE_REGISTRY,
    get_mx_dtype,
    mx_dtype,
    optimal_output_dtype,
)
from .dtypes import *  # noqa: F401,F403  (int4d, float4d, int8dh, ...)
from .checkpoint import load_quantized, save_quantized  # noqa: F401
from .dynamic import dynamic_quantize, fused_int8_linear, mx_dynamic_linear  # noqa: F401
from .fused import fused_linear_relu, fused_silu_and_mul  # noqa: F401
from .hadamard import sign_vector  # noqa: F401
from .kv_cache import kv_cache_quantizer  # noqa: F401
from .linear import mx_linear, to_mx  # noqa: F401
from .tensor import mx_matmul, mx_matmul_kmajor, mx_tensor, register_kernel  # noqa: F401

__version__ = "0.1.0"
