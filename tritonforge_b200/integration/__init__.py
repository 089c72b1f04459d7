"""Model integration: swap HF Qwen2 linear/norm/MLP pieces for the B200 kernels
(reference src/tritonforge/integration/__init__.py)."""

from __future__ import annotations

from .qwen import QuantLinear, patch_model  # noqa: F401

__all__ = ["QuantLinear", "patch_model"]
