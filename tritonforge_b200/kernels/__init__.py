"""B200 CUDA kernels behind the reference's ``tritonforge.kernels`` API
(src/tritonforge/kernels/__init__.py:5-9)."""

from __future__ import annotations

from .dequant_gemm import quantized_linear  # noqa: F401
from .rmsnorm_residual import rmsnorm, rmsnorm_residual  # noqa: F401
from .swiglu import swiglu  # noqa: F401

__all__ = ["quantized_linear", "rmsnorm", "rmsnorm_residual", "swiglu"]
