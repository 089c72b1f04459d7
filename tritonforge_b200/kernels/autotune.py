"""Launch-config vocabulary kept for drop-in compatibility.

The reference passes Triton block hints around as a ``ConfigDict``
(src/tritonforge/kernels/autotune.py:8-15) and picks defaults per M
(``default_dequant_config``, :47-51). The CUDA kernels here size their own
tiles, so block hints are accepted and ignored. One key means something:
``"regime"`` (``"auto"``, ``"gemv"``, ``"gemm"`` or ``"simt"``) pins the
quantized-linear kernel; tests and benchmarks use it to run each regime.
"""

from __future__ import annotations

from typing import TypedDict


class ConfigDict(TypedDict, total=False):
    BLOCK_M: int
    BLOCK_N: int
    BLOCK_K: int
    BLOCK_KH: int
    BLOCK: int
    num_warps: int
    num_stages: int
    regime: str


def default_dequant_config(m: int, block_m_hint: int | None = None) -> ConfigDict:
    """The default config for `m` rows: let the native dispatcher choose (it
    takes the decode GEMV up to 32 rows and the tcgen05 GEMM above when the
    shape and alignment allow, the generic kernel otherwise). The arguments
    keep the reference's signature."""
    return {"regime": "auto"}
