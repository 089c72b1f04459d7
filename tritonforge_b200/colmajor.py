"""Tiled column-major int4 weights for the decode engine.

The reference stores packed int4 codes K-major, ``packed [K_pad/2, N]``
(src/tritonforge/quant.py:25-63), and its decode path runs the same kernel as
prefill (src/tritonforge/kernels/dequant_gemm.py:121-210). A decode engine
that owns its weights can repack them once (``repack_cm``) into 16 KiB tiles
``[ceil(N/256), K_pad/128, 256, 64]`` (the codes of one output column
contiguous along k, ``tf_repack_int4_cm``) and run ``quantized_linear_cm``:
the tcgen05 decode kernel with the weights on the MMA's N = 256. Outputs equal
``kernels.quantized_linear`` on the original packing within the
floating-point contract (same dequantised weights, fp32 accumulation, same
roundings). Scales, zeros and bias keep their formats.
"""

from __future__ import annotations

import dataclasses

import torch

from . import _lib


TILE_COLS, TILE_K = 256, 128


def cm_shape(n: int, k_pad: int) -> tuple[int, int, int, int]:
    return (-(-n // TILE_COLS), k_pad // TILE_K, TILE_COLS, TILE_K // 2)


def repack_cm(packed: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """packed uint8 [K_pad/2, N] (reference format) -> tiles uint8 [ceil(N/256), K_pad/128, 256, 64]."""
    dev = _lib.require_cuda(packed)
    if packed.dtype != torch.uint8 or packed.dim() != 2:
        raise ValueError("packed must be a 2-D uint8 tensor")
    packed = packed.contiguous()
    half, n = packed.shape
    if (2 * half) % TILE_K:
        raise ValueError("packed K must be a multiple of 128")
    shape = cm_shape(n, 2 * half)
    if out is None:
        out = torch.empty(shape, dtype=torch.uint8, device=dev)
    if tuple(out.shape) != shape or out.dtype != torch.uint8 or not out.is_contiguous():
        raise ValueError(f"out must be a contiguous uint8 {shape} tensor")
    _lib.check(_lib.load().tf_repack_int4_cm(packed.data_ptr(), out.data_ptr(), n, 2 * half,
                                             _lib.stream_ptr(dev)), "repack_int4_cm")
    return out


def _check(x, packed_cm, scales, zeros):
    if x.dim() != 2 or packed_cm.dim() != 4 or scales.dim() != 2:
        raise ValueError("x must be 2-D, packed_cm [NB, S, 256, 64] (repack_cm), scales/zeros 2-D")
    if packed_cm.dtype != torch.uint8:
        raise ValueError("packed_cm must be uint8")
    n = scales.shape[1]
    if tuple(packed_cm.shape) != cm_shape(n, packed_cm.shape[1] * TILE_K):
        raise ValueError(f"packed_cm shape {tuple(packed_cm.shape)} does not match N={n}")
    if scales.dtype != x.dtype or zeros.dtype != x.dtype:
        raise ValueError("scales and zeros must have x's dtype")
    if x.stride(1) != 1 or not packed_cm.is_contiguous() or not scales.is_contiguous() or not zeros.is_contiguous():
        raise ValueError("x rows, packed_cm, scales and zeros must be contiguous")


def quantized_linear_cm(x: torch.Tensor, packed_cm: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor,
                        bias: torch.Tensor | None = None, group_size: int = 128, *,
                        out: torch.Tensor | None = None) -> torch.Tensor:
    """x [M, K] @ W (+ bias) with W given column-major (``repack_cm``); one
    kernel launch per 64 rows."""
    dev = _lib.require_cuda(x, packed_cm, scales, zeros, bias)
    _check(x, packed_cm, scales, zeros)
    m, k = x.shape
    n, half = scales.shape[1], packed_cm.shape[1] * TILE_K // 2
    if out is None:
        out = torch.empty((m, n), dtype=x.dtype, device=dev)
    ws = _lib.workspaces.get(dev, _lib.load().tf_qlinear_cm_workspace_bytes(m, n, 2 * half))
    _lib.check(_lib.load().tf_qlinear_cm(
        x.data_ptr(), x.stride(0), _lib.dtype_code(x.dtype), packed_cm.data_ptr(), scales.data_ptr(),
        zeros.data_ptr(), _lib.dtype_code(scales.dtype), _lib.ptr(bias),
        _lib.dtype_code(bias.dtype) if bias is not None else 0, out.data_ptr(), out.stride(0), m, n, k, 2 * half,
        group_size, ws.data_ptr(), ws.numel(), _lib.stream_ptr(dev)), "qlinear_cm")
    return out


def qlinear_cm_swiglu(x: torch.Tensor, packed_cm: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor,
                      group_size: int = 128, *, out: torch.Tensor | None = None) -> torch.Tensor:
    """silu(x @ Wg) * (x @ Wu) for gate/up interleaved per 64 columns,
    column-major; one kernel launch per 64 rows."""
    dev = _lib.require_cuda(x, packed_cm, scales, zeros)
    _check(x, packed_cm, scales, zeros)
    m, k = x.shape
    n, half = scales.shape[1], packed_cm.shape[1] * TILE_K // 2
    if out is None:
        out = torch.empty((m, n // 2), dtype=x.dtype, device=dev)
    ws = _lib.workspaces.get(dev, _lib.load().tf_qlinear_cm_workspace_bytes(m, n, 2 * half))
    _lib.check(_lib.load().tf_qlinear_cm_swiglu(
        x.data_ptr(), x.stride(0), _lib.dtype_code(x.dtype), packed_cm.data_ptr(), scales.data_ptr(),
        zeros.data_ptr(), _lib.dtype_code(scales.dtype), out.data_ptr(), out.stride(0), m, n, k, 2 * half,
        group_size, ws.data_ptr(), ws.numel(), _lib.stream_ptr(dev)), "qlinear_cm_swiglu")
    return out


@dataclasses.dataclass
class CMLinear:
    """An int4 linear held in the tiled column-major layout (``repack_cm``):
    the tiles replace ``QuantLinear.packed``; scales, zeros and bias keep the
    reference's formats ([K_pad/g, N], [N])."""

    tiles: torch.Tensor
    scales: torch.Tensor
    zeros: torch.Tensor
    in_features: int
    out_features: int
    bias: torch.Tensor | None = None
    group_size: int = 128

    @classmethod
    def from_quant(cls, ql) -> "CMLinear":
        """From a QuantLinear (or anything with packed/scales/zeros/bias/group_size)."""
        return cls(repack_cm(ql.packed), ql.scales.contiguous(), ql.zeros.contiguous(), ql.in_features,
                   ql.out_features, ql.bias, ql.group_size)

    def __call__(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        return quantized_linear_cm(x, self.tiles, self.scales, self.zeros, self.bias, self.group_size, out=out)
