"""CPU tests of the boundary: the C-ABI library loads and exports every entry
point the header declares, and the Python layer validates arguments exactly as
the reference does (ValueError) before touching a GPU; with no GPU the ops fail
loudly instead of falling back to the CPU."""

from __future__ import annotations

import ctypes
import pathlib
import re

import pytest
import torch

from tritonforge_b200 import _lib, kernels, quant
from tritonforge_b200.kernels.autotune import default_dequant_config

ROOT = pathlib.Path(__file__).resolve().parents[1]


def _declared_symbols() -> set[str]:
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = h.read_text()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names |= set(re.findall(r"\b(tf_[a-z0-9_]+)\s*\(", text))
    return names


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    declared = _declared_symbols()
    assert {"tf_qlinear", "tf_rmsnorm_residual", "tf_swiglu", "tf_quantize_int4"} <= declared
    for name in sorted(declared):
        assert hasattr(lib, name), f"{name} declared in include/ but not exported"
    assert declared <= set(_lib.SIGNATURES), "python binding misses a declared entry point"


def test_abi_version_and_status_strings():
    lib = _lib.load()
    assert lib.tf_abi_version() == 2
    assert lib.tf_status_string(0) == b"ok"
    assert lib.tf_status_string(_lib.ERR_WORKSPACE).startswith(b"workspace")
    assert lib.tf_status_string(99) == b"unknown status"


def test_workspace_sizes_are_sane():
    # decode shapes: split-K partial sums stay on chip (cluster reduction), the
    # workspace is the 256-byte header holding the device error word; the
    # prefill GEMM's stream-K schedule keeps up to two 256 x 256 fp32 partial
    # tiles per CTA (148 SMs without a GPU) after 512 bytes, and its arrival
    # counters (8 per tile, up to 2048 tiles) at the end
    lib = _lib.load()
    for m, n, k in [(1, 4864, 896), (16, 18944, 3584), (32, 8192, 29568), (128, 8192, 29568),
                    (2048, 18944, 3584), (2048, 3584, 3584)]:
        assert lib.tf_qlinear_workspace_bytes(m, n, k, 128) == 256
        assert lib.tf_qlinear_gemm_stream_k_grid(m, n, k) == 0
    for m, n, k in [(512, 3584, 18944), (300, 1008, 18944), (2048, 1280, 8192)]:
        grid = lib.tf_qlinear_gemm_stream_k_grid(m, n, k)
        assert 2 <= grid <= 148
        tiles = -(-n // 256) * -(-m // 256)
        partials = 2 * grid * 256 * 256 * 4
        assert tiles <= 2048
        assert lib.tf_qlinear_workspace_bytes(m, n, k, 128) == 512 + partials + 2048 * 32


def test_c_level_validation_without_gpu():
    """Argument checks in the library run before any CUDA call."""
    lib = _lib.load()
    rc = lib.tf_qlinear(None, 896, 7, None, None, None, 0, None, 0, None, 4864,
                        1, 4864, 896, 896, 128, None, 0, None)
    assert rc == _lib.ERR_BAD_DTYPE
    rc = lib.tf_qlinear(None, 896, 0, None, None, None, 0, None, 0, None, 4864,
                        1, 4864, 1000, 896, 128, None, 0, None)
    assert rc == _lib.ERR_BAD_SHAPE
    assert b"K=1000" in lib.tf_last_error_message()
    rc = lib.tf_qlinear(None, 896, 0, None, None, None, 0, None, 0, None, 4864,
                        1, 4864, 896, 900, 128, None, 0, None)
    assert rc == _lib.ERR_BAD_SHAPE
    # empty problems are valid no-ops
    assert lib.tf_qlinear(None, 0, 0, None, None, None, 0, None, 0, None, 1,
                          0, 1, 0, 128, 128, None, 0, None) == 0
    assert lib.tf_swiglu(None, None, None, 0, 0, None) == 0
    assert lib.tf_swiglu(None, None, None, 5, 9, None) in (_lib.ERR_BAD_ARG, _lib.ERR_BAD_DTYPE)
    assert lib.tf_quantize_int4(None, 4, 8, 3, None, None, None, 0, None) == _lib.ERR_BAD_ARG
    assert lib.tf_rmsnorm_residual(None, None, None, 0, None, None, 2, 8, ctypes.c_float(1e-6), 0,
                                   None) == _lib.ERR_BAD_ARG


# ---- Python-level validation: mirrors reference tests/test_kernels.py ----------

def _w(n=32, k=256):
    packed = torch.zeros(k // 2, n, dtype=torch.uint8)
    scales = torch.ones(k // 128, n, dtype=torch.float16)
    zeros = torch.zeros(k // 128, n, dtype=torch.float16)
    return packed, scales, zeros


def test_quantized_linear_rejects_bad_dtype():
    packed, scales, zeros = _w()
    x = torch.randn(4, 256, dtype=torch.float32)
    with pytest.raises(ValueError):
        kernels.quantized_linear(x, packed, scales, zeros)


@pytest.mark.parametrize("case", ["ndim", "packed_dtype", "group", "scales", "k_too_big"])
def test_quantized_linear_validation(case):
    packed, scales, zeros = _w()
    x = torch.randn(4, 256, dtype=torch.float16)
    kw = {}
    if case == "ndim":
        x = x.reshape(1, 4, 256)
    elif case == "packed_dtype":
        packed = packed.to(torch.int16)
    elif case == "group":
        kw["group_size"] = 96
    elif case == "scales":
        scales = scales[:1]
    elif case == "k_too_big":
        x = torch.randn(4, 300, dtype=torch.float16)
    with pytest.raises(ValueError):
        kernels.quantized_linear(x, packed, scales, zeros, **kw)


def test_rmsnorm_validation():
    x = torch.randn(4, 64, dtype=torch.float16)
    with pytest.raises(ValueError):
        kernels.rmsnorm_residual(x, torch.randn(4, 32, dtype=torch.float16), torch.randn(64))
    with pytest.raises(ValueError):
        kernels.rmsnorm(x, torch.randn(63))
    with pytest.raises(ValueError):
        kernels.rmsnorm(x.reshape(2, 2, 64), torch.randn(64))


def test_swiglu_shape_mismatch():
    with pytest.raises(ValueError):
        kernels.swiglu(torch.randn(4, 8), torch.randn(4, 9))


def test_quant_validation():
    with pytest.raises(ValueError):
        quant.quantize_int4_group(torch.zeros(8), 128)
    with pytest.raises(ValueError):
        quant.quantize_int4_group(torch.zeros(2, 8), 1)
    with pytest.raises(ValueError):
        quant.dequantize_int4(torch.zeros(64, 4, dtype=torch.uint8), torch.zeros(3, 4),
                              torch.zeros(3, 4), group_size=128)
    assert quant.padded_k(129, 128) == 256 and quant.padded_k(8, 1) == 8


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU behaviour")
def test_no_cpu_fallback():
    packed, scales, zeros = _w()
    x = torch.randn(4, 256, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="CUDA"):
        kernels.quantized_linear(x, packed, scales, zeros, config=default_dequant_config(4))
    with pytest.raises(RuntimeError, match="CUDA"):
        kernels.swiglu(torch.randn(4, 8, dtype=torch.float16), torch.randn(4, 8, dtype=torch.float16))
    with pytest.raises(RuntimeError, match="CUDA"):
        quant.quantize_int4_group(torch.randn(4, 128), 128)


def test_allreduce_rmsnorm_validates_without_a_gpu():
    lib = _lib.load()
    # null pointers / rank outside the group are rejected before anything is launched
    assert lib.tf_allreduce_rmsnorm_residual(None, None, 0, 64, 0, 2, None, None, None, _lib.BF16, None, None, 4,
                                             8192, 1e-6, _lib.BF16, _lib.F32, None, None) == _lib.ERR_BAD_ARG
    assert lib.tf_allreduce_rmsnorm_residual(None, None, 0, 64, 3, 2, None, None, None, _lib.BF16, None, None, 4,
                                             8192, 1e-6, _lib.BF16, _lib.F32, None, None) == _lib.ERR_BAD_SHAPE
    assert lib.tf_allreduce_rmsnorm_residual(None, None, 0, 64, 0, 2, None, None, None, _lib.BF16, None, None, 0,
                                             8192, 1e-6, _lib.BF16, _lib.F32, None, None) == _lib.OK


def test_colmajor_entry_points_validate_without_a_gpu():
    """The column-major decode entry points check their arguments before any
    CUDA call; the layout size is ceil(N/256)*256 x K_pad/2 bytes."""
    lib = _lib.load()
    assert lib.tf_int4_cm_bytes(4864, 896) == 19 * 256 * 448
    assert lib.tf_int4_cm_bytes(256, 128) == 256 * 64
    assert lib.tf_int4_cm_bytes(0, 128) == 0
    assert lib.tf_repack_int4_cm(None, None, 64, 200, None) == _lib.ERR_BAD_SHAPE  # K_pad % 128
    assert b"multiple of 128" in lib.tf_last_error_message()
    assert lib.tf_repack_int4_cm(None, None, -1, 128, None) == _lib.ERR_BAD_SHAPE
    assert lib.tf_repack_int4_cm(None, None, 64, 128, None) == _lib.ERR_BAD_ARG  # null pointers
    assert lib.tf_repack_int4_cm(None, None, 0, 128, None) == 0  # empty: no-op
    assert lib.tf_qlinear_cm_workspace_bytes(32, 8192, 8192) >= 256
    # rows not 16-byte aligned (ldx % 8 != 0) are outside the kernel's range:
    # rejected as unsupported before launching (any M runs, 64 rows per launch)
    x = ctypes.c_void_p(16)
    rc = lib.tf_qlinear_cm(x, 257, 1, x, x, x, 1, None, 0, x, 128, 65, 128, 256, 256, 128, x, 256, None)
    assert rc == _lib.ERR_UNSUPPORTED and b"aligned rows" in lib.tf_last_error_message()
    rc = lib.tf_qlinear_cm_swiglu(x, 256, 1, x, x, x, 1, x, 64, 4, 192, 256, 256, 128, x, 256, None)
    assert rc == _lib.ERR_BAD_SHAPE  # N % 128


def test_colmajor_python_layer_checks():
    from tritonforge_b200 import colmajor

    assert colmajor.cm_shape(4864, 896) == (19, 7, 256, 64)
    with pytest.raises(RuntimeError):  # no CPU path
        colmajor.repack_cm(torch.zeros(64, 256, dtype=torch.uint8))
