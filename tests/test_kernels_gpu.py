"""GPU parity: every CUDA kernel against the CPU oracle on identical seeded
inputs (shapes of the reference's own tests, of the 0.5B/7B/72B configurations,
and the edge cases), plus the committed golden vectors of the reference."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import ops as oops
from oracle import quant as oquant
from tests import golden_io as gio
from tests.parity import NP_DT, assert_rms_close, assert_swiglu_close, bits, f32, oracle_linear, oracle_quantize
from tritonforge_b200 import _lib, kernels, quant

pytestmark = pytest.mark.gpu
GROUP = 128
DTYPES = [torch.float16, torch.bfloat16]


def _linear_inputs(m, n, k, dtype, w_std=1.0, bias=True, seed=0, param_dtype=None):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=g).to(dtype).cuda()
    w = (torch.randn(n, k, generator=g) * w_std).cuda()
    packed, scales, zeros, _ = quant.quantize_int4_group(w, GROUP, param_dtype or dtype)
    b = torch.randn(n, generator=g).to(dtype).cuda() if bias else None
    return x, packed, scales, zeros, b


# ---- quantized_linear ------------------------------------------------------
REF_SHAPES = [(1, 64, 128), (1, 896, 896), (3, 127, 129), (16, 128, 256), (17, 64, 256),
              (64, 512, 896), (128, 256, 1024)]


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("m,n,k", REF_SHAPES)
def test_quantized_linear_reference_shapes(m, n, k, dtype):
    x, packed, scales, zeros, b = _linear_inputs(m, n, k, dtype)
    out = kernels.quantized_linear(x, packed, scales, zeros, b)
    ref = oracle_linear(x, packed, scales, zeros, b)
    assert_rms_close(out, ref, dtype, f"qlinear {m}x{n}x{k}")


DECODE_SHAPES = [(896, 4864), (4864, 896), (896, 896), (896, 128),
                 (3584, 3584), (3584, 512), (3584, 18944), (18944, 3584)]


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("k,n", DECODE_SHAPES)
@pytest.mark.parametrize("m", [1, 4, 8, 16, 32])
def test_gemv_decode_shapes(m, k, n, dtype):
    if m in (4, 32) and n * k > 30_000_000:
        pytest.skip("covered by the other M values at this size")
    x, packed, scales, zeros, b = _linear_inputs(m, n, k, dtype, w_std=0.02, bias=(n != 512), seed=m + n)
    out = kernels.quantized_linear(x, packed, scales, zeros, b, config={"regime": "gemv"})
    ref = oracle_linear(x, packed, scales, zeros, b)
    assert_rms_close(out, ref, dtype, f"gemv {m}x{n}x{k}")


@pytest.mark.parametrize("regime", ["gemv", "simt"])
@pytest.mark.parametrize("xdt,pdt", [(torch.bfloat16, torch.float16), (torch.float16, torch.bfloat16)])
def test_mixed_param_dtype(regime, xdt, pdt):
    # the reference's QuantLinear stores fp16 scales by default, also for bf16 models
    x, packed, scales, zeros, b = _linear_inputs(8, 4864, 896, xdt, w_std=0.02, param_dtype=pdt)
    b = b.to(pdt)
    out = kernels.quantized_linear(x, packed, scales, zeros, b, config={"regime": regime})
    ref = oracle_linear(x, packed, scales, zeros, b)
    assert_rms_close(out, ref, xdt, "mixed")


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("m,n,k", [(1, 4864, 896), (5, 896, 4864), (32, 512, 3584), (8, 256, 200),
                                   (3, 127, 129), (40, 4864, 896)])
def test_simt_regime(m, n, k, dtype):
    x, packed, scales, zeros, b = _linear_inputs(m, n, k, dtype, w_std=0.02, seed=7)
    out = kernels.quantized_linear(x, packed, scales, zeros, b, config={"regime": "simt"})
    ref = oracle_linear(x, packed, scales, zeros, b)
    assert_rms_close(out, ref, dtype, "simt", max_mismatch=0.02)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("k,regime", [(192, "gemv"), (200, "auto"), (1216, "gemv"), (1168, "auto")])
def test_x_shorter_than_packed_k(k, regime, dtype):
    # K < K_pad: the kernels read x[:, K:] as zeros (the reference pads x)
    x, packed, scales, zeros, b = _linear_inputs(4, 1024, k, dtype, w_std=0.02, seed=3)
    out = kernels.quantized_linear(x, packed, scales, zeros, b, config={"regime": regime})
    ref = oracle_linear(x, packed, scales, zeros, b)
    assert_rms_close(out, ref, dtype, f"K={k} < K_pad")


def test_no_bias_fp32_bias_and_strided_x():
    x, packed, scales, zeros, _ = _linear_inputs(4, 2048, 1024, torch.float16, w_std=0.02, seed=5)
    ref = oracle_linear(x, packed, scales, zeros, None)
    assert_rms_close(kernels.quantized_linear(x, packed, scales, zeros), ref, torch.float16, "no bias")
    b32 = torch.randn(2048, device="cuda")
    ref_b = oops.quantized_linear(f32(x), packed.cpu().numpy(), f32(scales), f32(zeros), f32(b32), GROUP,
                                  "float16")
    assert_rms_close(kernels.quantized_linear(x, packed, scales, zeros, b32), ref_b, torch.float16, "f32 bias")
    wide = torch.zeros(4, 1536, dtype=torch.float16, device="cuda")
    wide[:, :1024] = x
    out = kernels.quantized_linear(wide[:, :1024], packed, scales, zeros)  # row stride 1536
    assert_rms_close(out, ref, torch.float16, "strided x")


def test_empty_and_determinism():
    x, packed, scales, zeros, b = _linear_inputs(0, 512, 256, torch.float16)
    assert kernels.quantized_linear(x, packed, scales, zeros, b).shape == (0, 512)
    x, packed, scales, zeros, b = _linear_inputs(16, 3584, 18944, torch.bfloat16, w_std=0.02, seed=9)
    a1 = kernels.quantized_linear(x, packed, scales, zeros, b)
    a2 = kernels.quantized_linear(x, packed, scales, zeros, b)
    assert torch.equal(a1.view(torch.int16), a2.view(torch.int16)), "split-K reduction is not deterministic"
    ws = _lib.workspaces.get(x.device, 0)
    err = _lib.ctypes.c_int(0)
    rc = _lib.load().tf_workspace_error(ws.data_ptr(), _lib.ctypes.byref(err),
                                        _lib.stream_ptr(x.device))
    assert rc == 0 and err.value == 0


@pytest.mark.parametrize("dtype", DTYPES)
def test_large_m_rows_sampled(dtype):
    # prefill shape of the 7B config: check 64 sampled rows against the oracle
    m, k, n = 2048, 3584, 3584
    x, packed, scales, zeros, b = _linear_inputs(m, n, k, dtype, w_std=0.02, seed=11)
    out = kernels.quantized_linear(x, packed, scales, zeros, b)
    rows = torch.randperm(m, generator=torch.Generator().manual_seed(0))[:64].sort().values
    ref = oracle_linear(x[rows.cuda()], packed, scales, zeros, b)
    assert_rms_close(out[rows.cuda()], ref, dtype, "prefill rows")


def test_golden_linear_cases():
    rec = gio.load()
    for case in rec["linear/cases"]:
        case = str(case)
        dt = torch.float16 if gio.dtype_of(rec, f"{case}/x") == "float16" else torch.bfloat16
        x = torch.from_numpy(gio.get_f32(rec, f"{case}/x")).to(dt).cuda()
        packed = torch.from_numpy(gio.get(rec, f"{case}/packed")[0]).cuda()
        s = torch.from_numpy(gio.get_f32(rec, f"{case}/scales")).to(dt).cuda()
        z = torch.from_numpy(gio.get_f32(rec, f"{case}/zeros")).to(dt).cuda()
        b = (torch.from_numpy(gio.get_f32(rec, f"{case}/bias")).to(dt).cuda()
             if gio.has(rec, f"{case}/bias") else None)
        out = kernels.quantized_linear(x, packed, s, z, b)
        assert_rms_close(out, gio.get_f32(rec, f"{case}/out"), dt, case)


# ---- rmsnorm_residual / rmsnorm ---------------------------------------------
NORM_SHAPES = [(1, 896), (4, 896), (16, 1536), (128, 896), (1, 3584), (64, 3584), (2048, 3584),
               (1, 8192), (3, 100), (2, 16384), (1, 65544)]


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("m,n", NORM_SHAPES)
def test_rmsnorm_residual(m, n, dtype):
    g = torch.Generator().manual_seed(m + n)
    x = torch.randn(m, n, generator=g).to(dtype).cuda()
    r = torch.randn(m, n, generator=g).to(dtype).cuda()
    w = (1 + 0.02 * torch.randn(n, generator=g)).to(dtype).cuda()
    normed, summed = kernels.rmsnorm_residual(x, r, w)
    ref_n, ref_s = oops.rmsnorm_residual(f32(x), f32(r), f32(w), 1e-6, NP_DT[dtype])
    assert np.array_equal(f32(summed), ref_s), "summed must equal round(x + r) exactly"
    assert_rms_close(normed, ref_n, dtype, "normed", max_mismatch=0.01)
    plain = kernels.rmsnorm(x, w)
    assert_rms_close(plain, oops.rmsnorm(f32(x), f32(w), 1e-6, NP_DT[dtype]), dtype, "plain",
                     max_mismatch=0.01)


def test_rmsnorm_golden():
    rec = gio.load()
    for case in rec["rmsnorm/cases"]:
        case = str(case)
        dt = torch.float16 if gio.dtype_of(rec, f"{case}/x") == "float16" else torch.bfloat16
        t = {k: torch.from_numpy(gio.get_f32(rec, f"{case}/{k}")).to(dt).cuda() for k in "xrw"}
        normed, summed = kernels.rmsnorm_residual(t["x"], t["r"], t["w"])
        assert np.array_equal(bits(summed), gio.get(rec, f"{case}/summed")[0])
        assert_rms_close(normed, gio.get_f32(rec, f"{case}/normed"), dt, case, max_mismatch=0.02)
        assert_rms_close(kernels.rmsnorm(t["x"], t["w"]), gio.get_f32(rec, f"{case}/plain"), dt, case)


# ---- swiglu -------------------------------------------------------------------
@pytest.mark.parametrize("dtype", DTYPES + [torch.float32])
@pytest.mark.parametrize("shape", [(1, 4864), (3, 127), (16, 4864), (129, 4864), (64, 18944), (7,)])
def test_swiglu(shape, dtype):
    g = torch.Generator().manual_seed(sum(shape))
    gate = (torch.randn(*shape, generator=g) * 3).to(dtype).cuda()
    up = torch.randn(*shape, generator=g).to(dtype).cuda()
    out = kernels.swiglu(gate, up)
    ref = oops.swiglu(f32(gate), f32(up), NP_DT[dtype])
    assert_rms_close(out, ref, dtype, "swiglu", max_mismatch=0.01 if dtype != torch.float32 else None)


def test_swiglu_unaligned_and_golden():
    base_g = torch.randn(4097, dtype=torch.float16, device="cuda")
    base_u = torch.randn(4097, dtype=torch.float16, device="cuda")
    gate, up = base_g[1:], base_u[1:]  # 2-byte offset: scalar path
    ref = oops.swiglu(f32(gate), f32(up), "float16")
    assert_rms_close(kernels.swiglu(gate, up), ref, torch.float16, "unaligned", max_mismatch=0.01)
    rec = gio.load()
    for case in rec["swiglu/cases"]:
        case = str(case)
        dt = torch.float16 if gio.dtype_of(rec, f"{case}/g") == "float16" else torch.bfloat16
        gg = torch.from_numpy(gio.get_f32(rec, f"{case}/g")).to(dt).cuda()
        uu = torch.from_numpy(gio.get_f32(rec, f"{case}/u")).to(dt).cuda()
        assert_rms_close(kernels.swiglu(gg, uu), gio.get_f32(rec, f"{case}/out"), dt, case,
                         max_mismatch=0.01)


# ---- quantizer / unpack / dequant: bit-exact ------------------------------------
def test_quantizer_golden_bit_exact():
    rec = gio.load()
    for case in rec["quant/cases"]:
        p = f"quant/{case}"
        n, k, g, k_pad, is_bf16 = (int(v) for v in rec[f"{p}/meta"])
        dt = torch.bfloat16 if is_bf16 else torch.float16
        w = torch.from_numpy(gio.get(rec, f"{p}/w")[0]).cuda()
        packed, scales, zeros, kp = quant.quantize_int4_group(w, g, dt)
        assert kp == k_pad
        assert np.array_equal(packed.cpu().numpy(), gio.get(rec, f"{p}/packed")[0]), case
        assert np.array_equal(bits(scales), gio.get(rec, f"{p}/scales")[0]), case
        assert np.array_equal(bits(zeros), gio.get(rec, f"{p}/zeros")[0]), case
        assert np.array_equal(quant.unpack_int4(packed).cpu().numpy(), gio.get(rec, f"{p}/codes")[0])
        dense = quant.dequantize_int4(packed, scales, zeros, g, dt)
        assert np.array_equal(bits(dense), gio.get(rec, f"{p}/dense")[0]), case


@pytest.mark.parametrize("n,k,group,dtype,std", [
    (4864, 896, 128, torch.float16, 0.02), (896, 4864, 128, torch.bfloat16, 0.02),
    (1000, 300, 64, torch.float16, 1.0), (77, 1000, 256, torch.bfloat16, 0.5),
    (33, 130, 2, torch.float16, 1.0), (64, 96, 6, torch.float16, 1.0), (130, 1024, 512, torch.float16, 3.0)])
def test_quantizer_bit_exact_vs_oracle(n, k, group, dtype, std):
    w = torch.randn(n, k, generator=torch.Generator().manual_seed(n * k)) * std
    w[0, :group] = 0.0          # all-zero group: zero-point -0.0
    w[1, :] = 0.25              # constant row
    packed, scales, zeros, k_pad = quant.quantize_int4_group(w.cuda(), group, dtype)
    o_packed, o_scales, o_zeros, o_kpad = oracle_quantize(w, group, dtype)
    assert k_pad == o_kpad
    assert np.array_equal(packed.cpu().numpy(), o_packed)
    assert np.array_equal(bits(scales), o_scales)
    assert np.array_equal(bits(zeros), o_zeros)
    dense = quant.dequantize_int4(packed, scales, zeros, group, dtype)
    o_dense = oquant.dequantize_int4(o_packed, o_scales, o_zeros, group, NP_DT[dtype], NP_DT[dtype])
    assert np.array_equal(bits(dense), o_dense)


def test_quantize_cpu_input_round_trip_device():
    w = torch.randn(64, 256)
    packed, scales, zeros, _ = quant.quantize_int4_group(w, 128)
    assert packed.device.type == "cpu" and scales.device.type == "cpu"
    recon = quant.quantize_dequantize(w.cuda(), group_size=128)
    err = quant.quantization_error(w.cuda(), recon)
    assert err["max_abs"] < 0.3 and err["mean_abs"] < 0.12  # reference tests/test_quant.py:30-36


# ---- prefill regime (tcgen05 GEMM) -----------------------------------------
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("m,n,k", [(33, 128, 128), (64, 256, 896), (128, 128, 1024), (200, 384, 512),
                                   (512, 640, 640), (600, 144, 1152), (1100, 4864, 896)])
def test_gemm_regime(m, n, k, dtype):
    x, packed, scales, zeros, b = _linear_inputs(m, n, k, dtype, w_std=0.02, seed=m + k)
    out = kernels.quantized_linear(x, packed, scales, zeros, b, config={"regime": "gemm"})
    rows = torch.arange(m) if m <= 256 else torch.randperm(m, generator=torch.Generator().manual_seed(1))[:96].sort().values
    ref = oracle_linear(x[rows.cuda()], packed, scales, zeros, b)
    assert_rms_close(out[rows.cuda()], ref, dtype, f"gemm {m}x{n}x{k}")
    again = kernels.quantized_linear(x, packed, scales, zeros, b, config={"regime": "gemm"})
    assert torch.equal(out, again), "deterministic"


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("m,n,k", [(512, 3584, 18944), (300, 1008, 18944), (300, 256, 16384), (1024, 2048, 8192)])
def test_gemm_stream_k(m, n, k, dtype):
    """Shapes whose 256 x 256 tiles would leave SMs idle run the stream-K
    schedule (tiles split between CTAs, the pieces added in k order by the
    last CTA to arrive): sampled rows against the oracle, bit-identical across
    launches, and within the contract with a header-only workspace (which
    runs one tile per CTA)."""
    lib = _lib.load()
    assert lib.tf_qlinear_gemm_stream_k_grid(m, n, k) > 0
    x, packed, scales, zeros, b = _linear_inputs(m, n, k, dtype, w_std=0.02, seed=m + n)
    out = kernels.quantized_linear(x, packed, scales, zeros, b, config={"regime": "gemm"})
    rows = torch.randperm(m, generator=torch.Generator().manual_seed(2))[:64].sort().values
    rows = torch.cat([rows, torch.tensor([m - 1])]).unique().cuda()
    ref = oracle_linear(x[rows], packed, scales, zeros, b)
    pre = oracle_linear(x[rows], packed, scales, zeros, None)
    assert_rms_close(out[rows], ref, dtype, f"stream-K gemm {m}x{n}x{k}", pre_bias=pre)
    for _ in range(2):
        again = kernels.quantized_linear(x, packed, scales, zeros, b, config={"regime": "gemm"})
        assert torch.equal(out, again), "deterministic"
    ws = torch.zeros(256, dtype=torch.uint8, device="cuda")
    dp = torch.full_like(out, float("nan"))
    _lib.check(lib.tf_qlinear_ex(x.data_ptr(), x.stride(0), _lib.dtype_code(dtype), packed.data_ptr(),
                                 scales.data_ptr(), zeros.data_ptr(), _lib.dtype_code(dtype), b.data_ptr(),
                                 _lib.dtype_code(dtype), dp.data_ptr(), n, m, n, k, k, GROUP, ws.data_ptr(),
                                 ws.numel(), _lib.REGIME_GEMM, _lib.stream_ptr(x.device)), "qlinear_ex")
    assert_rms_close(dp[rows], ref, dtype, f"data-parallel gemm {m}x{n}x{k}", pre_bias=pre)
    assert torch.isfinite(dp).all()
    assert _lib.workspaces.errors(x.device) == 0 and int(ws[:4].view(torch.int32).item()) == 0


@pytest.mark.parametrize("m,n,k", [(512, 1024, 8192), (2048, 1280, 8192)])
def test_gemm_stream_k_partial_is_the_unrounded_sum(m, n, k):
    """tf_qlinear_partial (a row-parallel shard's fp32 partial) on the
    stream-K schedule: finite everywhere, and rounded once equal bit for bit
    to the regular entry point's output on the same schedule."""
    dtype = torch.bfloat16
    lib = _lib.load()
    assert lib.tf_qlinear_gemm_stream_k_grid(m, n, k) > 0
    x, packed, scales, zeros, _ = _linear_inputs(m, n, k, dtype, w_std=0.02, bias=False, seed=k)
    want = kernels.quantized_linear(x, packed, scales, zeros, None, GROUP)
    ws = _lib.workspaces.get(x.device, lib.tf_qlinear_workspace_bytes(m, n, k, GROUP))
    part = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
    _lib.check(lib.tf_qlinear_partial(x.data_ptr(), k, _lib.BF16, packed.data_ptr(), scales.data_ptr(),
                                      zeros.data_ptr(), _lib.BF16, part.data_ptr(), n, m, n, k, k, GROUP,
                                      ws.data_ptr(), ws.numel(), _lib.stream_ptr(x.device)), "qlinear_partial")
    torch.cuda.synchronize()
    assert torch.isfinite(part).all()
    assert torch.equal(part.to(dtype), want)
    rows = torch.tensor([0, m // 2, m - 1]).cuda()
    assert_rms_close(want[rows], oracle_linear(x[rows], packed, scales, zeros, None), dtype, "stream-K partial")


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("m,n,k", [(33, 512, 896), (64, 3584, 3584), (100, 256, 1024), (128, 896, 4864)])
def test_auto_regime_between_33_and_128_rows(m, n, k, dtype):
    """The automatic regime runs 33..128 rows as 32-row chunks of the decode
    GEMV: every row (the partial last chunk included) against the oracle, and
    each chunk equal to the decode GEMV on those rows alone."""
    x, packed, scales, zeros, b = _linear_inputs(m, n, k, dtype, w_std=0.02, seed=m + n)
    out = kernels.quantized_linear(x, packed, scales, zeros, b)
    ref = oracle_linear(x, packed, scales, zeros, b)
    assert_rms_close(out, ref, dtype, f"auto {m}x{n}x{k}")
    for r in range(0, m, 32):
        alone = kernels.quantized_linear(x[r:r + 32].contiguous(), packed, scales, zeros, b, config={"regime": "gemv"})
        assert torch.equal(out[r:r + 32], alone)


# ---- fused gate|up + SwiGLU (decode regime) --------------------------------
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("m,i,k", [(1, 4864, 896), (8, 4864, 896), (3, 896, 4864), (16, 18944, 3584),
                                   (32, 7424, 8192), (5, 1024, 29568), (40, 4864, 896), (200, 4864, 896),
                                   (300, 1024, 16384), (1100, 896, 4864)])
def test_qlinear_swiglu(m, i, k, dtype):
    """The fused gate|up + SwiGLU in every regime: the decode GEMV (M <= 32),
    its 32-row chunks (40), the GEMM's SwiGLU epilogue one tile per CTA (200,
    1100) and on the stream-K schedule (300 x 1024 x 16384), against the
    oracle's separately rounded projections."""
    from tritonforge_b200.tp import interleave_gate_up

    g = torch.Generator().manual_seed(m + i)
    x = torch.randn(m, k, generator=g).to(dtype).cuda()
    wg = (torch.randn(i, k, generator=g) * 0.02).cuda()
    wu = (torch.randn(i, k, generator=g) * 0.02).cuda()
    pg, sg, zg, _ = quant.quantize_int4_group(wg, GROUP, dtype)
    pu, su, zu, _ = quant.quantize_int4_group(wu, GROUP, dtype)
    packed = interleave_gate_up(pg, pu).contiguous()
    scales = interleave_gate_up(sg, su).contiguous()
    zeros = interleave_gate_up(zg, zu).contiguous()
    out = torch.full((m, i), float("nan"), dtype=dtype, device="cuda")
    need = _lib.load().tf_qlinear_workspace_bytes(m, 2 * i, packed.shape[0] * 2, GROUP)
    assert (m, i, k) != (300, 1024, 16384) or _lib.load().tf_qlinear_gemm_stream_k_grid(m, 2 * i, k) > 0
    ws = torch.zeros(max(need, 1 << 20), dtype=torch.uint8, device="cuda")
    rc = _lib.load().tf_qlinear_swiglu(x.data_ptr(), x.stride(0), _lib.dtype_code(dtype), packed.data_ptr(),
                                       scales.data_ptr(), zeros.data_ptr(), _lib.dtype_code(dtype), out.data_ptr(),
                                       out.stride(0), m, 2 * i, k, packed.shape[0] * 2, GROUP, ws.data_ptr(),
                                       ws.numel(), _lib.stream_ptr(x.device))
    _lib.check(rc, "qlinear_swiglu")
    gate = oracle_linear(x, pg, sg, zg, None)  # the separate projections, rounded to the dtype
    up = oracle_linear(x, pu, su, zu, None)
    assert_swiglu_close(out, gate, up, dtype, f"qlinear_swiglu {m}x{i}x{k}")
    assert int(ws[:4].view(torch.int32).item()) == 0
