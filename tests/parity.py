"""Parity helpers: compare CUDA outputs with the CPU oracle.

Tolerance (the contract for floating-point outputs): max-abs error
<= 1e-2 x RMS(oracle output) for fp16 and <= 2e-2 x RMS for bf16. Integer and
byte outputs (codes, packed nibbles, scale/zero bit patterns) must be equal.
"""

from __future__ import annotations

import numpy as np
import torch

from oracle import ops as oops
from oracle import quant as oquant

RMS_TOL = {torch.float16: 1e-2, torch.bfloat16: 2e-2, torch.float32: 1e-5}
NP_DT = {torch.float16: "float16", torch.bfloat16: "bfloat16", torch.float32: "float32"}


def f32(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def bits(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu().contiguous()
    if t.dtype in (torch.float16, torch.bfloat16):
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def assert_rms_close(out: torch.Tensor, ref: np.ndarray, dtype: torch.dtype, what: str = "",
                     max_mismatch: float | None = None, mean_frac: float | None = 0.1,
                     pre_bias: np.ndarray | None = None) -> dict:
    """Every element within the contract, max(RMS_TOL x RMS(ref), one ulp of
    the output type at ref): the contract is max-abs <= RMS_TOL x RMS, and a
    difference of one output ulp is the smallest nonzero difference there is
    (a bf16 output near 5 x RMS has an ulp of 2-3% of the RMS, so a single
    fp32 summation-order rounding flip of one large output would otherwise
    fail a correct kernel). Optionally at most `max_mismatch` of the elements
    differ from the oracle at all; the mean abs error is at most `mean_frac`
    of RMS_TOL x RMS (typical errors are ulp-level, not just bounded).
    `pre_bias` (the oracle's output before its bias add, rounded) allows one
    summation-order flip at that rounding point: out = round(round(acc) +
    bias) rounds twice, and a flip of round(acc) by one ulp of acc moves
    round(acc) + bias by that ulp and can also turn the second rounding the
    other way (round(acc) + bias is often a tie: two values of one binade add
    to one extra bit), so the output may differ by ulp(pre_bias) + ulp(out)."""
    got = f32(out)
    ref = np.asarray(ref, np.float32)
    assert got.shape == ref.shape, (got.shape, ref.shape)
    if got.size == 0:
        return {"max_abs": 0.0, "rms": 0.0}
    diff = np.abs(got.astype(np.float64) - ref.astype(np.float64))
    err = float(np.max(diff))
    rms = oops.rms(ref)
    tol = RMS_TOL[dtype] * rms
    assert np.isfinite(got).all(), f"{what}: non-finite output"
    mant = {torch.float16: 11, torch.bfloat16: 8, torch.float32: 24}[dtype]
    ulp = np.ldexp(1.0, np.frexp(np.abs(ref.astype(np.float64)) + 1e-30)[1] - mant)
    if pre_bias is not None:
        pre = np.asarray(pre_bias, np.float64)
        ulp = ulp + np.ldexp(1.0, np.frexp(np.abs(pre) + 1e-30)[1] - mant)
    bad = diff > np.maximum(tol, ulp)
    ulps = "1 ulp" if pre_bias is None else "1 ulp + 1 ulp before the bias"
    assert not bad.any(), (f"{what}: {int(bad.sum())} elements beyond max({RMS_TOL[dtype]} x RMS, {ulps}); "
                           f"max-abs {err:.4g}, RMS {rms:.4g}")
    mism = float(np.mean(got != ref))
    mean_err = float(np.mean(np.abs(got.astype(np.float64) - ref.astype(np.float64))))
    if mean_frac is not None:
        assert mean_err <= mean_frac * tol, f"{what}: mean abs error {mean_err:.4g} > {mean_frac} x {tol:.4g}"
    if max_mismatch is not None:
        assert mism <= max_mismatch, f"{what}: {mism:.3%} of elements differ from the oracle"
    return {"max_abs": err, "rms": rms, "mismatch": mism, "mean_abs": mean_err}


def oracle_linear(x: torch.Tensor, packed: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor,
                  bias: torch.Tensor | None, group: int = 128) -> np.ndarray:
    return oops.quantized_linear(f32(x), packed.cpu().numpy(), f32(scales), f32(zeros),
                                 None if bias is None else f32(bias), group, NP_DT[x.dtype])


def oracle_quantize(w: torch.Tensor, group: int, dtype: torch.dtype):
    return oquant.quantize_int4_group(w.detach().float().cpu().numpy(), group, NP_DT[dtype])


def assert_swiglu_close(out: torch.Tensor, gate: np.ndarray, up: np.ndarray, dtype: torch.dtype, what: str) -> None:
    """A fused gate|up + SwiGLU output against swiglu(gate, up) of the oracle's
    separately rounded projections. The kernel rounds gate and up exactly where
    the oracle does, but its fp32 accumulation order differs, so a projection
    may land one ulp away; the product then moves by that ulp times the other
    factor. Allowed per element: the contract's tolerance, or that one-ulp
    propagation plus one ulp of the output; the mean error stays at a tenth of
    the tolerance."""
    ref = oops.swiglu(gate, up, NP_DT[dtype])
    got = f32(out).astype(np.float64)
    assert np.isfinite(got).all(), f"{what}: non-finite output"
    g64, u64, r64 = gate.astype(np.float64), up.astype(np.float64), ref.astype(np.float64)
    mant = 11 if dtype == torch.float16 else 8

    def ulp(v):
        return np.ldexp(1.0, np.frexp(np.abs(v) + 1e-30)[1] - mant)

    sig = 1.0 / (1.0 + np.exp(-g64))
    dsilu = sig * (1.0 + g64 * (1.0 - sig))
    bound = np.abs(dsilu * u64) * ulp(g64) + np.abs(g64 * sig) * ulp(u64) + ulp(r64)
    err = np.abs(got - r64)
    tol = RMS_TOL[dtype] * oops.rms(ref)
    bad = (err > tol) & (err > bound)
    assert not bad.any(), f"{what}: {int(bad.sum())} outputs beyond tolerance, max {err.max():.4g}"
    assert err.mean() <= 0.1 * tol, f"{what}: mean error {err.mean():.4g}"
