"""CPU checks of the tiled column-major layout restatement in the oracle: it
holds the same codes as the reference's K-major packing, in the documented
order."""

from __future__ import annotations

import numpy as np

from oracle import quant as oquant


def test_repack_cm_round_trip_and_order():
    rng = np.random.default_rng(0)
    n, k_pad = 300, 256
    packed = rng.integers(0, 256, size=(k_pad // 2, n), dtype=np.uint8)
    tiles = oquant.repack_cm(packed)
    assert tiles.shape == (2, 2, 256, 64)
    assert np.array_equal(oquant.unpack_cm(tiles, n), oquant.unpack_int4(packed))
    assert not tiles[1, :, n - 256:].any(), "columns beyond N are zero"
    codes = oquant.unpack_int4(packed)
    col, s, w = 261, 1, 6  # block 1 row 5, stage 1, word 6 (chunk 1) -> stored chunk 1 ^ (5 // 2 % 4) = 3
    b, r = divmod(col, 256)
    chunk, e = divmod(w, 4)
    pos = 16 * (chunk ^ ((r // 2) % 4)) + 4 * e
    word = int.from_bytes(tiles[b, s, r, pos:pos + 4].tobytes(), "little")
    for p in range(4):
        assert (word >> (4 * p)) & 15 == codes[128 * s + 8 * w + 2 * p, col]
        assert (word >> (4 * p + 16)) & 15 == codes[128 * s + 8 * w + 2 * p + 1, col]


def test_colmajor_layers_converts_only_wide_projections(monkeypatch):
    """QwenWeights.colmajor_layers converts the projections with K >= 2048 to
    CMLinear in new layer dicts and leaves the caller's layers untouched (the
    GPU repack is stubbed out here)."""
    import torch

    from tritonforge_b200 import colmajor
    from tritonforge_b200.decode import QwenWeights
    from tritonforge_b200.integration.qwen import QuantLinear

    def fake_from_quant(cls, ql):
        return cls(torch.empty(0, dtype=torch.uint8), ql.scales, ql.zeros, ql.in_features, ql.out_features,
                   ql.bias, ql.group_size)

    monkeypatch.setattr(colmajor.CMLinear, "from_quant", classmethod(fake_from_quant))

    def ql(k, n=16):
        return QuantLinear(torch.zeros(k // 2, n, dtype=torch.uint8), torch.ones(k // 128, n),
                           torch.zeros(k // 128, n), k, n)

    layer = {"in_norm": torch.ones(8), "post_norm": torch.ones(8), "qkv": ql(2048), "o": ql(1024),
             "gu": ql(4096), "down": ql(1920)}
    w = QwenWeights([layer], torch.zeros(4, 8), torch.zeros(4, 8), torch.ones(8), 8, 8, 1, 1, 8, 1e-6, 1e6)
    out = w.colmajor_layers()
    assert isinstance(out[0]["qkv"], colmajor.CMLinear) and isinstance(out[0]["gu"], colmajor.CMLinear)
    assert isinstance(out[0]["o"], QuantLinear) and isinstance(out[0]["down"], QuantLinear)
    assert all(isinstance(w.layers[0][n], QuantLinear) for n in ("qkv", "o", "gu", "down"))
    assert out[0]["in_norm"] is layer["in_norm"]
