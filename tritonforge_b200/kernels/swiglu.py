"""Fused SwiGLU activation on B200: ``out = silu(gate) * up``.

Same signature and validation as the reference's ``tritonforge.kernels.swiglu``
(src/tritonforge/kernels/swiglu.py:36-57); computed in fp32 and rounded once to
the input dtype by ``tf_swiglu`` of the native library.
"""

from __future__ import annotations

import torch

from .. import _lib
from .autotune import ConfigDict


def swiglu(gate: torch.Tensor, up: torch.Tensor, config: ConfigDict | None = None, *,
           out: torch.Tensor | None = None) -> torch.Tensor:
    if gate.shape != up.shape:
        raise ValueError(f"gate/up shape mismatch: {tuple(gate.shape)} vs {tuple(up.shape)}")
    if up.dtype != gate.dtype:
        raise ValueError(f"gate/up dtype mismatch: {gate.dtype} vs {up.dtype}")
    if gate.dtype not in (torch.float16, torch.bfloat16, torch.float32):
        raise ValueError(f"unsupported dtype {gate.dtype}")
    dev = _lib.require_cuda(gate, up)
    gate = gate.contiguous()
    up = up.contiguous()
    if out is None:
        out = torch.empty_like(gate)
    rc = _lib.load().tf_swiglu(gate.data_ptr(), up.data_ptr(), out.data_ptr(), gate.numel(),
                               _lib.dtype_code(gate.dtype), _lib.stream_ptr(dev))
    _lib.check(rc, "swiglu")
    return out
