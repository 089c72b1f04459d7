"""CPU restatement of the reference PyTorch oracles (TEST ORACLE ONLY).

Follows ``src/tritonforge/reference.py`` of the reference, with its rounding
points. Inputs are fp32 numpy arrays that hold values representable in the
activation dtype; ``dtype`` ("float16" / "bfloat16") names the tensors' dtype in
the reference, and every place where the reference materialises a tensor of that
dtype is a rounding point here (``quant.round_to``).

* ``quantized_linear``  -> reference.py:21-36: weight dequantised and rounded to
  the activation dtype; ``x @ W`` accumulated in fp32 (torch's CPU half GEMM
  accumulates in fp32) and rounded; ``+ bias`` rounded again.
* ``rmsnorm_residual``  -> reference.py:39-50: ``summed = x + r`` (rounded);
  fp32 mean of squares of the rounded sum; ``rstd = rsqrt(var + eps)``;
  ``normed = round(round(summed * rstd) * weight)`` (two roundings).
* ``rmsnorm``           -> the plain form used by the reference's integration
  test (tests/test_integration.py:276-284): same as above with ``summed = x``.
* ``swiglu``            -> reference.py:53-57: fp32 ``silu(g) * u``, one rounding.
"""

from __future__ import annotations

import numpy as np

from .quant import F16, dequantize_int4_f32, round_to


def _f32(a) -> np.ndarray:
    return np.asarray(a, dtype=np.float32)


def quantized_linear(x, packed, scales, zeros, bias=None, group_size: int = 128,
                     dtype: str = F16) -> np.ndarray:
    """reference.py:21-36. ``scales``/``zeros`` are fp32 values of the stored
    parameters; returns fp32 values of the ``dtype`` output."""
    x = _f32(x)
    w = round_to(dequantize_int4_f32(packed, scales, zeros, group_size), dtype)
    k = x.shape[1]
    if w.shape[0] != k:
        w = w[:k]
    acc = x.astype(np.float64) @ w.astype(np.float64)
    out = round_to(acc.astype(np.float32), dtype)
    if bias is not None:
        out = round_to(out + _f32(bias)[None, :], dtype)
    return out


def _mean_sq_f32(s: np.ndarray) -> np.ndarray:
    return (np.square(s.astype(np.float64)).sum(-1, keepdims=True) / s.shape[-1]).astype(
        np.float32)


def rmsnorm_residual(x, residual, weight, eps: float = 1e-6, dtype: str = F16):
    """reference.py:39-50. Returns (normed, summed)."""
    summed = round_to(_f32(x) + _f32(residual), dtype)
    var = _mean_sq_f32(summed)
    rstd = np.float32(1.0) / np.sqrt(var + np.float32(eps))
    t = round_to(summed * rstd, dtype)
    normed = round_to(t * _f32(weight)[None, :], dtype)
    return normed, summed


def rmsnorm(x, weight, eps: float = 1e-6, dtype: str = F16) -> np.ndarray:
    """Plain RMSNorm with the oracle's two roundings (tests/test_integration.py:276-284)."""
    s = _f32(x)
    var = _mean_sq_f32(s)
    rstd = np.float32(1.0) / np.sqrt(var + np.float32(eps))
    t = round_to(s * rstd, dtype)
    return round_to(t * _f32(weight)[None, :], dtype)


def swiglu(gate, up, dtype: str = F16) -> np.ndarray:
    """reference.py:53-57: fp32 ``(g * sigmoid(g)) * u`` rounded once."""
    g = _f32(gate)
    u = _f32(up)
    with np.errstate(over="ignore"):
        sig = np.float32(1.0) / (np.float32(1.0) + np.exp(-g))
    return round_to((g * sig).astype(np.float32) * u, dtype)


def max_abs_error(a, b) -> float:
    """reference.py:64-65."""
    return float(np.max(np.abs(_f32(a) - _f32(b)))) if np.size(a) else 0.0


def rms(a) -> float:
    a = _f32(a)
    return float(np.sqrt(np.mean(np.square(a.astype(np.float64))))) if a.size else 0.0
