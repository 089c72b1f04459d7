"""tritonforge_b200: B200-native (sm_100a) int4 decode/prefill kernels.

A drop-in for the hot path of TritonForge: ``tritonforge_b200.kernels``
(quantized_linear, rmsnorm_residual, rmsnorm, swiglu), ``tritonforge_b200.quant``
(the K-major int4 group format) and ``tritonforge_b200.integration``
(QuantLinear, patch_model). The kernels are hand-written CUDA in
``libtritonforge_b200.so`` behind the C ABI of ``include/tritonforge_b200.h``;
there is no CPU fallback.
"""

from __future__ import annotations

__version__ = "0.1.0"

from .quant import (  # noqa: F401
    dequantize_int4,
    padded_k,
    quantization_error,
    quantize_dequantize,
    quantize_int4_group,
    unpack_int4,
)

__all__ = [
    "__version__",
    "dequantize_int4",
    "padded_k",
    "quantization_error",
    "quantize_dequantize",
    "quantize_int4_group",
    "unpack_int4",
]
