"""CPU tests of the on-disk weight cache: a save/load round trip returns the
same bits in the reference's tensor formats, tied embeddings stay tied, and
foreign or truncated directories are rejected."""

from __future__ import annotations

import json
import os

import pytest
import torch

from tritonforge_b200.decode import QwenWeights
from tritonforge_b200.integration.qwen import QuantLinear


def _ql(n, k, g, bias):
    packed = torch.randint(0, 256, (k // 2, n), generator=g, dtype=torch.uint8)
    scales = torch.rand(k // 128, n, generator=g).to(torch.bfloat16)
    zeros = torch.randint(0, 16, (k // 128, n), generator=g).to(torch.bfloat16)
    b = torch.randn(n, generator=g).to(torch.bfloat16) if bias else None
    return QuantLinear(packed, scales, zeros, k, n, b, 128)


def _tiny(tied: bool) -> QwenWeights:
    g = torch.Generator().manual_seed(0)
    H, I, hq, hkv, D, V = 256, 384, 4, 2, 64, 1000
    layers = []
    for _ in range(2):
        layers.append({"in_norm": torch.randn(H, generator=g).to(torch.bfloat16),
                       "post_norm": torch.randn(H, generator=g).to(torch.bfloat16),
                       "qkv": _ql((hq + 2 * hkv) * D, H, g, True), "o": _ql(H, hq * D, g, False),
                       "gu": _ql(2 * I, H, g, False), "down": _ql(H, I, g, False)})
    embed = torch.randn(V, H, generator=g).to(torch.bfloat16)
    lm_head = embed if tied else torch.randn(V, H, generator=g).to(torch.bfloat16)
    return QwenWeights(layers, embed, lm_head, torch.ones(H, dtype=torch.bfloat16), H, I, hq, hkv, D, 1e-6, 1e6)


@pytest.mark.parametrize("tied", [True, False])
def test_round_trip_is_bit_exact(tmp_path, tied):
    w = _tiny(tied)
    w.save(str(tmp_path))
    r = QwenWeights.load(str(tmp_path), device="cpu")
    assert (r.hidden, r.inter, r.q_heads, r.kv_heads, r.head_dim, r.eps, r.rope_theta) == \
        (w.hidden, w.inter, w.q_heads, w.kv_heads, w.head_dim, w.eps, w.rope_theta)
    assert (r.lm_head is r.embed) == tied
    assert torch.equal(r.embed.view(torch.int16), w.embed.view(torch.int16))
    assert torch.equal(r.lm_head.view(torch.int16), w.lm_head.view(torch.int16))
    for a, b in zip(w.layers, r.layers):
        for n in ("in_norm", "post_norm"):
            assert torch.equal(a[n].view(torch.int16), b[n].view(torch.int16))
        for n in ("qkv", "o", "gu", "down"):
            qa, qb = a[n], b[n]
            assert torch.equal(qa.packed, qb.packed)
            assert torch.equal(qa.scales.view(torch.int16), qb.scales.view(torch.int16))
            assert torch.equal(qa.zeros.view(torch.int16), qb.zeros.view(torch.int16))
            assert (qa.bias is None) == (qb.bias is None)
            if qa.bias is not None:
                assert torch.equal(qa.bias.view(torch.int16), qb.bias.view(torch.int16))
            assert (qa.in_features, qa.out_features, qa.group_size) == (qb.in_features, qb.out_features,
                                                                        qb.group_size)
    man = json.load(open(tmp_path / "manifest.json"))
    assert all(e["offset"] % 256 == 0 for e in man["tensors"].values())


def test_rejects_foreign_and_truncated(tmp_path):
    w = _tiny(True)
    w.save(str(tmp_path))
    man = json.load(open(tmp_path / "manifest.json"))
    bad = dict(man, format="something-else")
    json.dump(bad, open(tmp_path / "manifest.json", "w"))
    with pytest.raises(ValueError, match="not a"):
        QwenWeights.load(str(tmp_path), device="cpu")
    json.dump(man, open(tmp_path / "manifest.json", "w"))
    # a shard of another tensor-parallel degree or rank is refused
    with pytest.raises(ValueError, match="wanted tp=2"):
        QwenWeights.load(str(tmp_path), device="cpu", tp=2, rank=0)
    with pytest.raises(ValueError, match="rank=1"):
        QwenWeights.load(str(tmp_path), device="cpu", tp=1, rank=1)
    QwenWeights.load(str(tmp_path), device="cpu", tp=1, rank=0)
    # another layout of the fused projections is refused
    json.dump(dict(man, layout={"gu": "gate then up"}), open(tmp_path / "manifest.json", "w"))
    with pytest.raises(ValueError, match="another layout"):
        QwenWeights.load(str(tmp_path), device="cpu")
    json.dump(man, open(tmp_path / "manifest.json", "w"))
    # a blob that does not belong to its manifest (an interrupted save) is refused
    size = os.path.getsize(tmp_path / "tensors.bin")
    with open(tmp_path / "tensors.bin", "r+b") as f:
        f.truncate(size - 100)
    with pytest.raises(ValueError, match="does not match its manifest"):
        QwenWeights.load(str(tmp_path), device="cpu")
    # a manifest that claims the short blob still stops at the tensor that runs past the end
    json.dump(dict(man, blob_bytes=size - 100), open(tmp_path / "manifest.json", "w"))
    with pytest.raises(ValueError, match="past the end"):
        QwenWeights.load(str(tmp_path), device="cpu")
