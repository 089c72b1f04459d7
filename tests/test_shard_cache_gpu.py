"""GPU test of the on-disk weight cache: a decoder built from saved-and-loaded
int4 shards produces bit-identical logits to one built from the originals."""

from __future__ import annotations

import pytest
import torch

from tritonforge_b200.decode import QwenDecoder, QwenWeights

pytestmark = pytest.mark.gpu


def test_loaded_weights_decode_identically(tmp_path):
    dev = torch.device("cuda", 0)
    w = QwenWeights.synthetic("7b", tp=2, rank=1, dtype=torch.bfloat16, device=dev, seed=7, layers=1)
    w.save(str(tmp_path))
    r = QwenWeights.load(str(tmp_path), device=dev)
    a, b = QwenDecoder(w, 4, 64), QwenDecoder(r, 4, 64)
    for d in (a, b):
        d.fill_cache(20, seed=3)
    for _ in range(2):
        a.step()
        b.step()
        assert torch.equal(a.buf["logits"], b.buf["logits"])
        assert torch.equal(a.tokens, b.tokens)
