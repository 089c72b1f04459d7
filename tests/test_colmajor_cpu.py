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
