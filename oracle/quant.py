"""Numpy restatement of the reference int4 group quantizer (TEST ORACLE ONLY).

Follows ``src/tritonforge/quant.py`` of the reference:

* ``padded_k``               -> quant.py:25-26
* ``quantize_int4_group``    -> quant.py:29-63
* ``unpack_int4``            -> quant.py:66-74
* ``dequantize_int4``        -> quant.py:77-105 (``_group_expand`` + dequant)
* ``repack_cm`` / ``unpack_cm`` -> the decode engine's tiled column-major layout of
  the same codes (no reference counterpart)

Format (the drop-in contract): for a weight ``W[N, K]`` (``nn.Linear`` layout)
K is zero-padded to ``K_pad`` (a multiple of the group size ``g``). Per
(column ``n``, group ``G``) of ``g`` consecutive k::

    scale = max((max - min) / 15, 1e-8)          # fp32, IEEE division
    zero  = clamp(rint(-min / scale), 0, 15)     # round-half-even
    code  = clamp(rint(w / scale + zero), 0, 15)

Codes are computed with the fp32 scale; the stored scale is the fp32 scale
rounded to the parameter dtype (fp16 or bf16). Codes are stored K-major, two per
byte: ``packed[j, n] = code[2j, n] | code[2j+1, n] << 4``. Scales and zeros are
stored ``[G, N]``. ``torch.clamp`` keeps ``-0.0`` (an all-zero group stores a
zero-point of ``-0.0``); this module keeps it too.

Half-precision values are carried as ``uint16`` bit patterns so that bf16 (which
numpy lacks) is handled exactly.
"""

from __future__ import annotations

import numpy as np

F16 = "float16"
BF16 = "bfloat16"


# --------------------------------------------------------------------------
# bit-level half conversions (round to nearest even)
# --------------------------------------------------------------------------
def f32_to_half_bits(x: np.ndarray, dtype: str) -> np.ndarray:
    """fp32 -> fp16/bf16 bit patterns, round-to-nearest-even."""
    x = np.asarray(x, dtype=np.float32)
    if dtype == F16:
        return x.astype(np.float16).view(np.uint16)
    if dtype == BF16:
        u = x.view(np.uint32).astype(np.uint64)
        is_nan = np.isnan(x)
        rounded = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
        return np.where(is_nan, np.uint16(0x7FC0), rounded).astype(np.uint16)
    raise ValueError(f"unsupported half dtype {dtype}")


def half_bits_to_f32(bits: np.ndarray, dtype: str) -> np.ndarray:
    bits = np.asarray(bits, dtype=np.uint16)
    if dtype == F16:
        return bits.view(np.float16).astype(np.float32)
    if dtype == BF16:
        return (bits.astype(np.uint32) << 16).view(np.float32)
    raise ValueError(f"unsupported half dtype {dtype}")


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round fp32 values to ``dtype`` and return them as fp32."""
    if dtype == "float32":
        return np.asarray(x, dtype=np.float32)
    return half_bits_to_f32(f32_to_half_bits(x, dtype), dtype)


def _clamp_keep_sign(v: np.ndarray, lo: float, hi: float) -> np.ndarray:
    # torch.clamp(v, lo, hi) == min(max(v, lo), hi) with "keep v when equal":
    # clamp(-0.0, 0, 15) stays -0.0.
    v = np.where(v < np.float32(lo), np.float32(lo), v)
    v = np.where(v > np.float32(hi), np.float32(hi), v)
    return v.astype(np.float32)


# --------------------------------------------------------------------------
# quant.py restatement
# --------------------------------------------------------------------------
def padded_k(k: int, group_size: int) -> int:
    """quant.py:25-26."""
    g = max(group_size, 2)
    return -(-k // g) * g


def quantize_int4_group(weight: np.ndarray, group_size: int = 128, dtype: str = F16):
    """quant.py:29-63. Returns (packed u8 [K_pad/2, N], scales bits u16 [G, N],
    zeros bits u16 [G, N], K_pad)."""
    w = np.asarray(weight, dtype=np.float32)
    if w.ndim != 2:
        raise ValueError(f"expected 2-D weight, got shape {w.shape}")
    if group_size < 2:
        raise ValueError("group_size must be >= 2")
    n, k = w.shape
    k_pad = padded_k(k, group_size)
    if k_pad != k:
        w = np.concatenate([w, np.zeros((n, k_pad - k), np.float32)], axis=1)
    groups = k_pad // group_size
    wg = w.reshape(n, groups, group_size)
    w_min = wg.min(axis=-1)
    w_max = wg.max(axis=-1)
    scale = (w_max - w_min).astype(np.float32) / np.float32(15.0)
    scale = np.where(scale < np.float32(1e-8), np.float32(1e-8), scale).astype(np.float32)
    zero = _clamp_keep_sign(np.rint((-w_min) / scale).astype(np.float32), 0.0, 15.0)
    q = wg / scale[..., None]
    q = (q + zero[..., None]).astype(np.float32)
    q = _clamp_keep_sign(np.rint(q).astype(np.float32), 0.0, 15.0)
    q = q.reshape(n, k_pad).astype(np.uint8)
    even = np.ascontiguousarray(q[:, 0::2].T)
    odd = np.ascontiguousarray(q[:, 1::2].T)
    packed = (even | (odd << 4)).astype(np.uint8)
    scales = f32_to_half_bits(np.ascontiguousarray(scale.T), dtype)
    zeros = f32_to_half_bits(np.ascontiguousarray(zero.T), dtype)
    return packed, scales, zeros, k_pad


def unpack_int4(packed: np.ndarray, k: int | None = None) -> np.ndarray:
    """quant.py:66-74: K-major packed [K_pad/2, N] -> codes [K_pad, N]."""
    packed = np.asarray(packed, dtype=np.uint8)
    if packed.ndim != 2:
        raise ValueError("packed must be 2-D")
    half, n = packed.shape
    out = np.empty((half * 2, n), np.uint8)
    out[0::2] = packed & 0x0F
    out[1::2] = (packed >> 4) & 0x0F
    return out if k is None else out[:k]


CM_COLS = 256  # columns of a tile of the tiled column-major layout
CM_K = 128     # k of a tile


def repack_cm(packed: np.ndarray) -> np.ndarray:
    """Tiled column-major layout used by the decode engine (a layout of the
    same codes, no reference counterpart): packed [K_pad/2, N] -> uint8
    [ceil(N/256), K_pad/128, 256, 64]. Tile (b, s) row r is column 256 b + r,
    k = 128 s .. 128 s + 127: little-endian 32-bit word w holds k = 8w..8w+7 of
    the tile with nibble p = code[8w + 2p] and nibble p + 4 = code[8w + 2p + 1]
    (p = 0..3); 16-byte chunk c of the row is stored at c ^ ((r // 2) % 4).
    Columns >= N are zero."""
    codes = unpack_int4(packed).astype(np.uint32)  # [K_pad, N]
    kp, n = codes.shape
    if kp % CM_K:
        raise ValueError("K_pad must be a multiple of 128")
    nb = -(-n // CM_COLS)
    full = np.zeros((kp, nb * CM_COLS), np.uint32)
    full[:, :n] = codes
    c = full.T.reshape(nb, CM_COLS, kp // CM_K, 16, 8)  # [block, row, stage, word, k in word]
    words = np.zeros(c.shape[:4], np.uint32)
    for p in range(4):
        words |= c[..., 2 * p] << (4 * p)
        words |= c[..., 2 * p + 1] << (4 * p + 16)
    words = words.transpose(0, 2, 1, 3)  # [block, stage, row, word]
    chunks = words.reshape(nb, kp // CM_K, CM_COLS, 4, 4)  # 16-byte chunks of 4 words
    out = np.empty_like(chunks)
    rows = np.arange(CM_COLS)
    for ch in range(4):
        out[:, :, rows, ch ^ ((rows // 2) % 4)] = chunks[:, :, rows, ch]
    return out.astype("<u4").view(np.uint8).reshape(nb, kp // CM_K, CM_COLS, 64)


def unpack_cm(tiles: np.ndarray, n: int) -> np.ndarray:
    """Inverse of ``repack_cm``: tiles [NB, S, 256, 64] -> codes [K_pad, n]."""
    t = np.ascontiguousarray(tiles, dtype=np.uint8)
    nb, ns = t.shape[:2]
    chunks = t.view("<u4").reshape(nb, ns, CM_COLS, 4, 4).astype(np.uint32)
    rows = np.arange(CM_COLS)
    logical = np.empty_like(chunks)
    for ch in range(4):
        logical[:, :, rows, ch] = chunks[:, :, rows, ch ^ ((rows // 2) % 4)]
    words = logical.reshape(nb, ns, CM_COLS, 16)
    codes = np.empty((nb, ns, CM_COLS, 16, 8), np.uint8)
    for p in range(4):
        codes[..., 2 * p] = (words >> (4 * p)) & 15
        codes[..., 2 * p + 1] = (words >> (4 * p + 16)) & 15
    # [block, stage, row, k in stage] -> [k, column]
    k_major = codes.reshape(nb, ns, CM_COLS, CM_K).transpose(1, 3, 0, 2).reshape(ns * CM_K, nb * CM_COLS)
    return k_major[:, :n].copy()


def dequantize_int4_f32(packed, scales_f32, zeros_f32, group_size: int = 128) -> np.ndarray:
    """quant.py:90-105 before the final cast: fp32 ``(code - zero) * scale``."""
    half, n = packed.shape
    k_pad = half * 2
    if k_pad % group_size != 0:
        raise ValueError(f"K_pad={k_pad} must be a multiple of group_size={group_size}")
    groups = k_pad // group_size
    s = np.asarray(scales_f32, np.float32)
    z = np.asarray(zeros_f32, np.float32)
    if s.shape != (groups, n) or z.shape != (groups, n):
        raise ValueError(f"expected group params [G, N] = [{groups}, {n}]")
    codes = unpack_int4(packed).astype(np.float32)
    s_full = np.repeat(s, group_size, axis=0)
    z_full = np.repeat(z, group_size, axis=0)
    return ((codes - z_full) * s_full).astype(np.float32)


def dequantize_int4(packed, scales_bits, zeros_bits, group_size: int = 128,
                    param_dtype: str = F16, dtype: str = F16) -> np.ndarray:
    """quant.py:90-105: dense K-major weight [K_pad, N] as ``dtype`` bit patterns
    (``float32`` returns fp32 values)."""
    s = half_bits_to_f32(scales_bits, param_dtype)
    z = half_bits_to_f32(zeros_bits, param_dtype)
    w = dequantize_int4_f32(packed, s, z, group_size)
    if dtype == "float32":
        return w
    return f32_to_half_bits(w, dtype)
