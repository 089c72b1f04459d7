"""GPU tests of the engine's prompt prefill (QwenDecoder.prefill_tokens): the
prefill against the same prompt fed through the decode step one token at a
time (same weights, the same kernels but for the summation order and the
attention library), at a length that runs the chunked decode GEMV (40 rows)
and one that runs the tcgen05 GEMM (200 rows)."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("batch,length", [(2, 40), (1, 200)])
def test_prefill_matches_token_by_token_decode(batch, length):
    from tests.parity import assert_rms_close, f32
    from tests.tp_check import logits_close, near_tie
    from tritonforge_b200.decode import QwenDecoder, QwenWeights

    dev = torch.device("cuda", 0)
    w = QwenWeights.synthetic("7b", dtype=torch.bfloat16, device=dev, seed=3, layers=2)
    a = QwenDecoder(w, batch, length + 16, colmajor=False)
    b = QwenDecoder(w, batch, length + 16, colmajor=False)
    g = torch.Generator().manual_seed(length)
    prompt = torch.randint(0, w.embed.shape[0], (batch, length), generator=g)
    got = a.prefill_tokens(prompt)
    b.pos.copy_(torch.tensor([0, 1], dtype=torch.int32))
    for t in range(length):
        b.tokens.copy_(prompt[:, t].to(dev))
        b.step()
    torch.cuda.synchronize()
    assert a.pos.tolist() == b.pos.tolist() == [length, length + 1]
    ok, err, rms, mean = logits_close(a.buf["logits"], b.buf["logits"])
    assert ok, f"last-position logits: max beyond one ulp {err:.4g}, mean {mean:.4g}, RMS {rms:.4g}"
    tie_ok, gap = near_tie(b.buf["logits"], b.tokens, got.to(dev), rms)
    assert tie_ok, f"greedy tokens differ beyond a near tie (gap {gap:.4g})"
    # the caches hold the same keys and values: the first layer's within the
    # per-op contract (identical inputs; the projections' fp32 sums differ in
    # order only), later layers within the whole-decode bound (their inputs
    # already carry the earlier layers' one-ulp flips)
    for li in range(len(w.layers)):
        for name, ca, cb in (("k", a.k_cache, b.k_cache), ("v", a.v_cache, b.v_cache)):
            got, want = ca[li, :, :, :length], cb[li, :, :, :length]
            if li == 0:
                assert_rms_close(got, f32(want), torch.bfloat16, f"{name} cache layer 0", mean_frac=None)
            else:
                ok, err, rms, mean = logits_close(got, want)
                assert ok, f"{name} cache layer {li}: max beyond one ulp {err:.4g}, mean {mean:.4g}, RMS {rms:.4g}"
    # both continue decoding from the prefilled state
    b.tokens.copy_(a.tokens)
    for _ in range(2):
        a.step()
        b.step()
        ok, err, rms, mean = logits_close(a.buf["logits"], b.buf["logits"])
        assert ok, f"decode after prefill: max beyond one ulp {err:.4g}, mean {mean:.4g}"
        b.tokens.copy_(a.tokens)
    assert a.device_errors() == 0 and b.device_errors() == 0


def test_prefill_needs_k_major_projections():
    from tritonforge_b200.decode import QwenDecoder, QwenWeights

    w = QwenWeights.synthetic("7b", dtype=torch.bfloat16, device=torch.device("cuda", 0), seed=3, layers=1)
    d = QwenDecoder(w, 16, 64)  # batches 9..64: column-major projections
    with pytest.raises(RuntimeError, match="K-major"):
        d.prefill_tokens(torch.zeros(16, 8, dtype=torch.long))
