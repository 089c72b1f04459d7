"""Readers for the committed golden vectors (``tests/golden/*.npz``)."""

from __future__ import annotations

import functools
import pathlib

import numpy as np

GOLDEN = pathlib.Path(__file__).resolve().parent / "golden"

_DT = {"f16": "float16", "bf16": "bfloat16"}


@functools.lru_cache(maxsize=None)
def load(name: str = "kernels_golden.npz") -> dict:
    with np.load(GOLDEN / name) as z:
        return {k: z[k] for k in z.files}


def get(rec: dict, name: str):
    """Return (array, tag) where tag is f16/bf16/f32/u8; half arrays are bits."""
    for tag in ("f16", "bf16", "f32", "u8"):
        key = f"{name}__{tag}"
        if key in rec:
            return rec[key], tag
    raise KeyError(name)


def get_f32(rec: dict, name: str) -> np.ndarray:
    """Array as fp32 values (half bit patterns decoded)."""
    from oracle.quant import half_bits_to_f32

    arr, tag = get(rec, name)
    if tag in _DT:
        return half_bits_to_f32(arr, _DT[tag])
    return arr.astype(np.float32) if tag == "f32" else arr


def dtype_of(rec: dict, name: str) -> str:
    _, tag = get(rec, name)
    return _DT.get(tag, tag)


def has(rec: dict, name: str) -> bool:
    return any(f"{name}__{t}" in rec for t in ("f16", "bf16", "f32", "u8"))
