"""Pin the CPU oracle against golden vectors recorded from the reference itself.

The quantizer, packer, unpacker and dequantizer must match bit for bit; the
floating-point oracles must match the reference's outputs exactly or within one
unit in the last place of the output dtype (the reference's CPU GEMM and mean
use a different summation order than the oracle).
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import ops, quant
from tests import golden_io as gio

REC = gio.load()


def _ulp_close(a: np.ndarray, b: np.ndarray, dtype: str, ulps: float = 1.0) -> bool:
    a = a.astype(np.float64)
    b = b.astype(np.float64)
    mant = 10 if dtype == "float16" else 7
    scale = np.maximum(np.abs(b), 6.1e-5 if dtype == "float16" else 1e-30)
    ulp = 2.0 ** (np.floor(np.log2(scale)) - mant)
    return bool(np.all(np.abs(a - b) <= ulps * ulp + 1e-12))


@pytest.mark.parametrize("case", [str(c) for c in REC["quant/cases"]])
def test_quantizer_bit_exact(case):
    p = f"quant/{case}"
    n, k, g, k_pad, is_bf16 = (int(v) for v in REC[f"{p}/meta"])
    dt = "bfloat16" if is_bf16 else "float16"
    w, _ = gio.get(REC, f"{p}/w")
    packed, scales, zeros, kp = quant.quantize_int4_group(w, g, dt)
    assert kp == k_pad == quant.padded_k(k, g)
    ref_packed, _ = gio.get(REC, f"{p}/packed")
    ref_scales, _ = gio.get(REC, f"{p}/scales")
    ref_zeros, _ = gio.get(REC, f"{p}/zeros")
    assert packed.shape == ref_packed.shape == (k_pad // 2, n)
    assert np.array_equal(packed, ref_packed)
    assert np.array_equal(scales, ref_scales)  # bit patterns, incl. sign of zero
    assert np.array_equal(zeros, ref_zeros)


@pytest.mark.parametrize("case", [str(c) for c in REC["quant/cases"]])
def test_unpack_and_dequant_bit_exact(case):
    p = f"quant/{case}"
    n, k, g, k_pad, is_bf16 = (int(v) for v in REC[f"{p}/meta"])
    dt = "bfloat16" if is_bf16 else "float16"
    packed, _ = gio.get(REC, f"{p}/packed")
    scales, _ = gio.get(REC, f"{p}/scales")
    zeros, _ = gio.get(REC, f"{p}/zeros")
    codes, _ = gio.get(REC, f"{p}/codes")
    assert np.array_equal(quant.unpack_int4(packed), codes)
    dense = quant.dequantize_int4(packed, scales, zeros, g, dt, dt)
    ref_dense, _ = gio.get(REC, f"{p}/dense")
    assert np.array_equal(dense, ref_dense)


def test_known_answer_pack():
    packed, _ = gio.get(REC, "kat/packed")
    codes, _ = gio.get(REC, "kat/codes")
    expect = np.array([[0, 1, 2, 3, 4, 5, 6, 7], [8, 9, 10, 11, 12, 13, 14, 15]], np.uint8).T
    assert np.array_equal(codes, expect)
    assert np.array_equal(quant.unpack_int4(packed), expect)


def test_padding_rows_dequantize_to_zero():
    packed, _ = gio.get(REC, "quant/pad_4x129/packed")
    scales, _ = gio.get(REC, "quant/pad_4x129/scales")
    zeros, _ = gio.get(REC, "quant/pad_4x129/zeros")
    dense = quant.dequantize_int4(packed, scales, zeros, 128, "float16", "float32")
    assert dense.shape == (256, 4)
    assert np.all(np.abs(dense[129:]) <= 1e-6)


def test_all_zero_group_keeps_negative_zero_point():
    zeros, _ = gio.get(REC, "quant/layout_zero/zeros")
    assert np.all(zeros == 0x8000)
    z_bits = quant.quantize_int4_group(np.zeros((2, 128), np.float32), 128)[2]
    assert np.all(z_bits == 0x8000)


def test_invalid_group_params_raise():
    packed = np.zeros((64, 4), np.uint8)
    with pytest.raises(ValueError):
        quant.dequantize_int4_f32(packed, np.zeros((3, 4)), np.zeros((3, 4)), 128)
    with pytest.raises(ValueError):
        quant.quantize_int4_group(np.zeros((2, 8), np.float32), 1)


@pytest.mark.parametrize("case", [str(c) for c in REC["linear/cases"]])
def test_linear_oracle_matches_reference(case):
    dt = gio.dtype_of(REC, f"{case}/x")
    x = gio.get_f32(REC, f"{case}/x")
    packed, _ = gio.get(REC, f"{case}/packed")
    s = gio.get_f32(REC, f"{case}/scales")
    z = gio.get_f32(REC, f"{case}/zeros")
    bias = gio.get_f32(REC, f"{case}/bias") if gio.has(REC, f"{case}/bias") else None
    out = ops.quantized_linear(x, packed, s, z, bias, 128, dt)
    ref = gio.get_f32(REC, f"{case}/out")
    assert out.shape == ref.shape
    # The reference's GEMM sums in a different order; allow one ulp of the
    # un-biased result plus one of the biased result.
    assert _ulp_close(out, ref, dt, ulps=2.0), ops.max_abs_error(out, ref)
    mism = np.mean(out != ref)
    assert mism < 0.05, mism


@pytest.mark.parametrize("case", [str(c) for c in REC["rmsnorm/cases"]])
def test_rmsnorm_oracle_matches_reference(case):
    dt = gio.dtype_of(REC, f"{case}/x")
    x = gio.get_f32(REC, f"{case}/x")
    r = gio.get_f32(REC, f"{case}/r")
    w = gio.get_f32(REC, f"{case}/w")
    normed, summed = ops.rmsnorm_residual(x, r, w, 1e-6, dt)
    assert np.array_equal(summed, gio.get_f32(REC, f"{case}/summed"))
    assert _ulp_close(normed, gio.get_f32(REC, f"{case}/normed"), dt, ulps=1.0)
    plain = ops.rmsnorm(x, w, 1e-6, dt)
    assert _ulp_close(plain, gio.get_f32(REC, f"{case}/plain"), dt, ulps=1.0)


@pytest.mark.parametrize("case", [str(c) for c in REC["swiglu/cases"]])
def test_swiglu_oracle_matches_reference(case):
    dt = gio.dtype_of(REC, f"{case}/g")
    g = gio.get_f32(REC, f"{case}/g")
    u = gio.get_f32(REC, f"{case}/u")
    out = ops.swiglu(g, u, dt)
    ref = gio.get_f32(REC, f"{case}/out")
    assert _ulp_close(out, ref, dt, ulps=1.0)
    assert np.mean(out != ref) < 0.01
