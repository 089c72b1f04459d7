"""GPU parity of the column-major decode path: tf_repack_int4_cm against the
oracle's restatement of the layout (bit-exact), and tf_qlinear_cm /
tf_qlinear_cm_swiglu (tcgen05; weights on the MMA's N, tokens on its M)
against the oracle's quantized_linear on the original K-major packing."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import quant as oquant
from tests.parity import assert_rms_close, assert_swiglu_close, f32, oracle_linear
from tritonforge_b200 import _lib, colmajor, kernels, quant
from tritonforge_b200.tp import interleave_gate_up

pytestmark = pytest.mark.gpu
DTYPES = [torch.float16, torch.bfloat16]


@pytest.mark.parametrize("n,k_pad", [(16, 128), (200, 1024), (896, 896), (4864, 29568), (300, 256)])
def test_repack_cm_bit_exact(n, k_pad):
    g = torch.Generator().manual_seed(n + k_pad)
    packed = torch.randint(0, 256, (k_pad // 2, n), generator=g, dtype=torch.uint8)
    got = colmajor.repack_cm(packed.cuda()).cpu().numpy()
    assert np.array_equal(got, oquant.repack_cm(packed.numpy()))


def _inputs(m, n, k, dtype, group=128, bias=True, seed=0, w_std=0.02):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=g).to(dtype).cuda()
    w = (torch.randn(n, k, generator=g) * w_std).cuda()
    packed, scales, zeros, _ = quant.quantize_int4_group(w, group, dtype)
    b = torch.randn(n, generator=g).to(dtype).cuda() if bias else None
    return x, packed, scales, zeros, b


CM_SHAPES = [(1, 128, 128), (1, 896, 896), (3, 4864, 896), (16, 1152, 3584), (17, 256, 1024), (5, 1024, 1216),
             (2, 64, 256), (32, 8192, 8192), (9, 8192, 29568), (32, 1280, 8192), (33, 1024, 2048), (64, 896, 896),
             (48, 3584, 18944), (4, 32768, 384), (2, 4096, 128), (100, 3584, 3584), (128, 1024, 2048),
             (65, 512, 8192)]


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("m,n,k", CM_SHAPES)
def test_qlinear_cm(m, n, k, dtype):
    x, packed, scales, zeros, b = _inputs(m, n, k, dtype, bias=(m % 2 == 1), seed=m * 7 + n)
    pcm = colmajor.repack_cm(packed)
    out = colmajor.quantized_linear_cm(x, pcm, scales, zeros, b)
    ref = oracle_linear(x, packed, scales, zeros, b)
    assert_rms_close(out, ref, dtype, f"qlinear_cm {m}x{n}x{k}")
    again = colmajor.quantized_linear_cm(x, pcm, scales, zeros, b)
    assert torch.equal(out, again), "deterministic: split blocks are added in a fixed order"
    # no bounded wait expired
    ws = _lib.workspaces.get(x.device, 0)
    assert int(ws[:4].view(torch.int32).item()) == 0


@pytest.mark.parametrize("dtype", DTYPES)
def test_qlinear_cm_group256_strided_x_out(dtype):
    m, n, k = 4, 512, 2048
    x, packed, scales, zeros, _ = _inputs(m, n, k, dtype, group=256, bias=False, seed=3)
    pcm = colmajor.repack_cm(packed)
    xs = torch.zeros(m, k + 64, dtype=dtype, device="cuda")
    xs[:, :k] = x
    out = torch.full((m, n + 32), float("nan"), dtype=dtype, device="cuda")
    colmajor.quantized_linear_cm(xs[:, :k], pcm, scales, zeros, None, 256, out=out[:, :n])
    ref = oracle_linear(x, packed, scales, zeros, None, group=256)
    assert_rms_close(out[:, :n], ref, dtype, "qlinear_cm group 256")
    assert torch.isnan(out[:, n:]).all(), "no write beyond N"


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("m,i,k", [(1, 4864, 896), (8, 4864, 896), (3, 896, 4864), (16, 18944, 3584),
                                   (32, 7424, 8192), (5, 1024, 29568), (4, 960, 1024), (64, 1024, 2048),
                                   (6, 16384, 384), (100, 1024, 2048)])
def test_qlinear_cm_swiglu(m, i, k, dtype):
    g = torch.Generator().manual_seed(m + i)
    x = torch.randn(m, k, generator=g).to(dtype).cuda()
    wg = (torch.randn(i, k, generator=g) * 0.02).cuda()
    wu = (torch.randn(i, k, generator=g) * 0.02).cuda()
    pg, sg, zg, _ = quant.quantize_int4_group(wg, 128, dtype)
    pu, su, zu, _ = quant.quantize_int4_group(wu, 128, dtype)
    pcm = colmajor.repack_cm(interleave_gate_up(pg, pu).contiguous())
    scales = interleave_gate_up(sg, su).contiguous()
    zeros = interleave_gate_up(zg, zu).contiguous()
    out = torch.full((m, i), float("nan"), dtype=dtype, device="cuda")
    colmajor.qlinear_cm_swiglu(x, pcm, scales, zeros, out=out)
    gate = oracle_linear(x, pg, sg, zg, None)
    up = oracle_linear(x, pu, su, zu, None)
    assert_swiglu_close(out, gate, up, dtype, f"qlinear_cm_swiglu {m}x{i}x{k}")


def test_qlinear_cm_rejects_unsupported():
    x, packed, scales, zeros, _ = _inputs(65, 128, 256, torch.bfloat16, bias=False)
    pcm = colmajor.repack_cm(packed)
    odd = torch.zeros(65, 257, dtype=torch.bfloat16, device="cuda")[:, :256]  # rows not 16-byte aligned
    odd.copy_(x)
    with pytest.raises(RuntimeError, match="qlinear_cm"):
        colmajor.quantized_linear_cm(odd, pcm, scales, zeros)
    with pytest.raises(ValueError):
        colmajor.quantized_linear_cm(x[:4].half(), pcm, scales, zeros)


@pytest.mark.parametrize("batch", [16, 48, 100])
def test_decoder_colmajor_matches_kmajor(batch):
    """The decode engine on tiled column-major weights (tcgen05 kernel) against
    the same engine on the reference's K-major packing (mma.sync / GEMM
    kernels): same weights, caches and tokens, logits within the
    tensor-parallel tolerance (a different fp32 summation order moves bf16
    roundings by an ulp), the same launches per step or fewer."""
    from tests.tp_check import logits_close
    from tritonforge_b200.colmajor import CMLinear
    from tritonforge_b200.decode import QwenDecoder, QwenWeights
    from tritonforge_b200.integration.qwen import QuantLinear

    w = QwenWeights.synthetic("7b", dtype=torch.bfloat16, device=torch.device("cuda", 0), seed=5, layers=2)
    a = QwenDecoder(w, batch, 96, colmajor=False)
    b = QwenDecoder(w, batch, 96)  # batch 9..128: column-major by default
    assert isinstance(a.layers[0]["qkv"], QuantLinear) and isinstance(w.layers[0]["gu"], QuantLinear)
    assert all(isinstance(b.layers[0][n], CMLinear) for n in ("qkv", "o", "gu", "down"))
    per = -(-batch // 64)  # launches per projection and per lm_head + argmax: one per 64 rows
    assert b.launches_per_step() == (3 + 4 * per) * 2 + 2 + per  # + embedding gather, first norm
    for d in (a, b):
        d.fill_cache(40, seed=2)
    for _ in range(3):
        a.step()
        b.step()
        ok, err, rms, mean = logits_close(b.buf["logits"], a.buf["logits"])
        assert ok, f"logits differ: max beyond one ulp {err:.4g}, mean {mean:.4g}, RMS {rms:.4g}"
        b.tokens.copy_(a.tokens)  # continue both on one token stream
    # the captured graph replays the same step
    saved = (b.tokens.clone(), b.pos.clone(), b.k_cache.clone(), b.v_cache.clone())
    eager = b.step().clone()
    b.tokens.copy_(saved[0]); b.pos.copy_(saved[1]); b.k_cache.copy_(saved[2]); b.v_cache.copy_(saved[3])
    assert torch.equal(b.replay().clone(), eager)


@pytest.mark.parametrize("layout,regime,m", [("kmajor", "gemv", 1), ("kmajor", "gemv", 16), ("kmajor", "gemv", 32),
                                              ("kmajor", "gemm", 160), ("kmajor", "simt", 5), ("cm", "cm", 1),
                                              ("cm", "cm", 32), ("cm", "cm", 64)])
def test_qlinear_partial_is_the_unrounded_sum(layout, regime, m):
    """tf_qlinear_partial / tf_qlinear_cm_partial (a row-parallel shard's fp32
    partial): the fp32 sums of the same kernel, not rounded, no bias. Rounded
    once they equal the regular entry point's output bit for bit; against a
    float64 sum of the oracle's dequantised weights they are fp32-accurate."""
    dtype = torch.bfloat16
    k, n = 2048, 1024
    g = torch.Generator().manual_seed(m + 7)
    x = torch.randn(m, k, generator=g).to(dtype).cuda()
    w = (torch.randn(n, k, generator=g) * 0.02).cuda()
    packed, scales, zeros, _ = quant.quantize_int4_group(w, 128, dtype)
    lib = _lib.load()
    ws = _lib.workspaces.get(x.device, 256)
    part = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
    if layout == "cm":
        tiles = colmajor.repack_cm(packed)
        want = colmajor.quantized_linear_cm(x, tiles, scales, zeros)
        rc = lib.tf_qlinear_cm_partial(x.data_ptr(), k, _lib.BF16, tiles.data_ptr(), scales.data_ptr(),
                                       zeros.data_ptr(), _lib.BF16, part.data_ptr(), n, m, n, k, k, 128,
                                       ws.data_ptr(), ws.numel(), _lib.stream_ptr(x.device))
    else:
        want = kernels.quantized_linear(x, packed, scales, zeros, None, 128, {"regime": regime})
        if regime == "gemv":
            rc = lib.tf_qlinear_partial(x.data_ptr(), k, _lib.BF16, packed.data_ptr(), scales.data_ptr(),
                                        zeros.data_ptr(), _lib.BF16, part.data_ptr(), n, m, n, k, k, 128,
                                        ws.data_ptr(), ws.numel(), _lib.stream_ptr(x.device))
        else:
            # the partial entry point picks its regime like tf_qlinear; force the others by shape:
            # simt through an odd stride (ldx not a multiple of 8), gemm through M > 128
            xs = x
            if regime == "simt":
                xs = torch.zeros(m, k + 1, dtype=dtype, device="cuda")[:, :k]
                xs.copy_(x)
            rc = lib.tf_qlinear_partial(xs.data_ptr(), xs.stride(0), _lib.BF16, packed.data_ptr(),
                                        scales.data_ptr(), zeros.data_ptr(), _lib.BF16, part.data_ptr(), n, m, n, k,
                                        k, 128, ws.data_ptr(), ws.numel(), _lib.stream_ptr(x.device))
    _lib.check(rc, "qlinear_partial")
    torch.cuda.synchronize()
    assert torch.isfinite(part).all()
    assert torch.equal(part.to(dtype), want), "rounded partial differs from the regular entry point"
    deq = oquant.round_to(oquant.dequantize_int4_f32(packed.cpu().numpy(), f32(scales), f32(zeros), 128), "bfloat16")
    exact = f32(x).astype(np.float64) @ np.asarray(deq, np.float64)[:k]
    err = np.abs(f32(part).astype(np.float64) - exact).max()
    assert err <= 1e-5 * np.abs(exact).max(), err
    assert _lib.workspaces.errors(x.device) == 0
