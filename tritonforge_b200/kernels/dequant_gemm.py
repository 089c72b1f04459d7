"""Fused int4 (group-wise, K-major packed) dequant + GEMM on B200.

``y = x @ dequant(packed) + bias`` with the reference's weight layout
(``packed[k//2, n]``, scales/zeros ``[G, N]``). Same signature, validation and
error behaviour as the reference's ``tritonforge.kernels.quantized_linear``
(src/tritonforge/kernels/dequant_gemm.py:121-210); the work runs in
``tf_qlinear`` of the native library, which picks the decode GEMV (M <= 32) or a
larger-M kernel itself.
"""

from __future__ import annotations

import torch

from .. import _lib
from .autotune import ConfigDict


def _validate(x: torch.Tensor, packed: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor,
              group_size: int) -> tuple[int, int, int]:
    """Reference dequant_gemm.py:121-148 (same checks, same messages)."""
    if x.ndim != 2:
        raise ValueError(f"x must be 2-D, got {tuple(x.shape)}")
    if x.dtype not in (torch.float16, torch.bfloat16):
        raise ValueError(f"x dtype must be fp16/bf16, got {x.dtype}")
    if packed.dtype != torch.uint8:
        raise ValueError(f"packed must be uint8, got {packed.dtype}")
    k_half, n = packed.shape
    k_pad = k_half * 2
    if k_pad % group_size != 0:
        raise ValueError(f"packed K={k_pad} not a multiple of group_size={group_size}")
    groups = k_pad // group_size
    if scales.shape != (groups, n) or zeros.shape != (groups, n):
        raise ValueError(
            f"scales/zeros must be [G, N] = [{groups}, {n}], "
            f"got {tuple(scales.shape)}/{tuple(zeros.shape)}"
        )
    if x.shape[1] > k_pad:
        raise ValueError(f"x has K={x.shape[1]} > packed K={k_pad}")
    return x.shape[0], n, k_pad


def workspace_bytes(m: int, n: int, k_pad: int, group_size: int = 128) -> int:
    return int(_lib.load().tf_qlinear_workspace_bytes(m, n, k_pad, group_size))


def quantized_linear(
    x: torch.Tensor,
    packed: torch.Tensor,
    scales: torch.Tensor,
    zeros: torch.Tensor,
    bias: torch.Tensor | None = None,
    group_size: int = 128,
    config: ConfigDict | None = None,
    *,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """Fused int4 dequant + GEMM. ``config`` block hints are accepted and ignored
    (``config["regime"]`` pins the kernel); ``out`` reuses a preallocated
    ``[M, N]`` output (no allocation, for CUDA-graph capture)."""
    m, n, k_pad = _validate(x, packed, scales, zeros, group_size)
    if scales.dtype not in (torch.float16, torch.bfloat16, torch.float32) or zeros.dtype != scales.dtype:
        raise ValueError(f"scales/zeros must share a float dtype, got {scales.dtype}/{zeros.dtype}")
    if bias is not None and bias.numel() == 0:
        bias = None
    if bias is not None and bias.numel() != n:
        raise ValueError(f"bias must have {n} elements, got {bias.numel()}")
    dev = _lib.require_cuda(x, packed, scales, zeros, bias)
    lib = _lib.load()
    if x.stride(1) != 1 or x.stride(0) < x.shape[1]:
        x = x.contiguous()
    packed = packed.contiguous()
    scales = scales.contiguous()
    zeros = zeros.contiguous()
    if bias is not None:
        bias = bias.contiguous()
        if bias.dtype not in (torch.float16, torch.bfloat16, torch.float32):
            bias = bias.float()
    if out is None:
        out = torch.empty((m, n), device=dev, dtype=x.dtype)
    elif out.shape != (m, n) or out.dtype != x.dtype or out.device != dev or out.stride(1) != 1:
        raise ValueError("out must be a [M, N] row-major tensor of x's dtype on x's device")
    if m == 0 or n == 0:
        return out
    regime = _lib.REGIMES[(config or {}).get("regime", "auto")]
    need = int(lib.tf_qlinear_workspace_bytes(m, n, k_pad, group_size))
    ws = _lib.workspaces.get(dev, need)
    rc = lib.tf_qlinear_ex(
        x.data_ptr(), x.stride(0), _lib.dtype_code(x.dtype),
        packed.data_ptr(), scales.data_ptr(), zeros.data_ptr(), _lib.dtype_code(scales.dtype),
        _lib.ptr(bias), _lib.dtype_code(bias.dtype) if bias is not None else 0,
        out.data_ptr(), out.stride(0),
        m, n, x.shape[1], k_pad, group_size,
        ws.data_ptr(), ws.numel(), regime, _lib.stream_ptr(dev))
    _lib.check(rc, "quantized_linear")
    return out
