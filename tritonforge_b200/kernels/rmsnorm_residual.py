"""Fused residual-add + RMSNorm (and plain RMSNorm) on B200.

Same signatures, validation and return values as the reference's
``tritonforge.kernels.rmsnorm_residual`` / ``rmsnorm``
(src/tritonforge/kernels/rmsnorm_residual.py:85-161); the work runs in
``tf_rmsnorm_residual`` of the native library (one pass over HBM, row kept in
registers).
"""

from __future__ import annotations

import torch

from .. import _lib
from .autotune import ConfigDict


def _launch(x: torch.Tensor, residual: torch.Tensor | None, weight: torch.Tensor, eps: float,
            write_sum: bool, normed: torch.Tensor | None = None,
            summed: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor | None]:
    # validation: reference rmsnorm_residual.py:93-98
    if x.ndim != 2:
        raise ValueError(f"expected 2-D input, got {tuple(x.shape)}")
    if weight.ndim != 1 or weight.shape[0] != x.shape[1]:
        raise ValueError(f"weight must be 1-D of length {x.shape[1]}")
    if residual is not None and residual.shape != x.shape:
        raise ValueError(f"residual shape {tuple(residual.shape)} != x {tuple(x.shape)}")
    if x.dtype not in (torch.float16, torch.bfloat16):
        raise ValueError(f"x dtype must be fp16/bf16, got {x.dtype}")
    if residual is not None and residual.dtype != x.dtype:
        raise ValueError(f"residual dtype {residual.dtype} != x dtype {x.dtype}")
    dev = _lib.require_cuda(x, residual, weight)
    x = x.contiguous()
    r = None if residual is None else residual.contiguous()
    weight = weight.contiguous()
    if weight.dtype not in (torch.float16, torch.bfloat16, torch.float32):
        weight = weight.float()
    m, n = x.shape
    if normed is None:
        normed = torch.empty_like(x)
    if write_sum and summed is None:
        summed = torch.empty_like(x)
    rc = _lib.load().tf_rmsnorm_residual(
        x.data_ptr(), _lib.ptr(r), weight.data_ptr(), _lib.dtype_code(weight.dtype),
        normed.data_ptr(), summed.data_ptr() if write_sum else None,
        m, n, float(eps), _lib.dtype_code(x.dtype), _lib.stream_ptr(dev))
    _lib.check(rc, "rmsnorm_residual" if residual is not None else "rmsnorm")
    return normed, (summed if write_sum else None)


def rmsnorm_residual(
    x: torch.Tensor,
    residual: torch.Tensor,
    weight: torch.Tensor,
    eps: float = 1e-6,
    config: ConfigDict | None = None,
    *,
    out: tuple[torch.Tensor, torch.Tensor] | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Returns (norm(x + residual), x + residual)."""
    normed, summed = _launch(x, residual, weight, eps, True,
                             *(out if out is not None else (None, None)))
    assert summed is not None
    return normed, summed


def rmsnorm(
    x: torch.Tensor,
    weight: torch.Tensor,
    eps: float = 1e-6,
    config: ConfigDict | None = None,
    *,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    normed, _ = _launch(x, None, weight, eps, False, out)
    return normed
