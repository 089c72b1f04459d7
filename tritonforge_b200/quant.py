"""Group-wise int4 quantization with the reference's K-major packed layout.

Same API and format as the reference's ``src/tritonforge/quant.py``:
``packed[j, n]`` holds the codes for k = 2j (low nibble) and 2j+1 (high
nibble); scales and zeros are ``[K_pad/g, N]``. The quantizer, unpacker and
dequantizer run as CUDA kernels (``tf_quantize_int4``, ``tf_unpack_int4``,
``tf_dequantize_int4``); the quantizer is bit-exact with the reference run on
the CPU (IEEE fp32 division, round-half-even, the sign of zero that
``torch.clamp`` keeps).

Tensors on the CPU are staged through the current CUDA device and the results
are returned on the input's device, as the reference returns them on the
weight's device. Without a CUDA device these functions raise.
"""

from __future__ import annotations

import torch

from . import _lib

LOW_MASK = 0x0F


def _ceil_div(a: int, b: int) -> int:
    return -(-a // b)


def padded_k(k: int, group_size: int) -> int:
    """Reference quant.py:25-26."""
    return _ceil_div(k, max(group_size, 2)) * max(group_size, 2)


def _cuda_device(t: torch.Tensor) -> torch.device:
    if t.is_cuda:
        return t.device
    if not torch.cuda.is_available():
        raise RuntimeError("tritonforge_b200.quant runs on CUDA only; no CUDA device is available")
    return torch.device("cuda", torch.cuda.current_device())


def quantize_int4_group(
    weight: torch.Tensor,
    group_size: int = 128,
    dtype: torch.dtype = torch.float16,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, int]:
    """Quantize a 2-D weight [N, K] into the K-major int4 layout (quant.py:29-63).

    Returns (packed [K_pad/2, N] uint8, scales [G, N] dtype, zeros [G, N] dtype,
    K_pad), K_pad = K rounded up to a multiple of group_size.
    """
    if weight.ndim != 2:
        raise ValueError(f"expected 2-D weight, got shape {tuple(weight.shape)}")
    if group_size < 2:
        raise ValueError("group_size must be >= 2")
    if group_size % 2 != 0:
        raise ValueError("group_size must be even (codes are packed in pairs along K)")
    if dtype not in (torch.float16, torch.bfloat16, torch.float32):
        raise ValueError(f"unsupported parameter dtype {dtype}")
    n, k = weight.shape
    k_pad = padded_k(k, group_size)
    dev = _cuda_device(weight)
    w = weight.detach().to(device=dev, dtype=torch.float32).contiguous()
    groups = k_pad // group_size
    packed = torch.empty((k_pad // 2, n), dtype=torch.uint8, device=dev)
    scales = torch.empty((groups, n), dtype=dtype, device=dev)
    zeros = torch.empty((groups, n), dtype=dtype, device=dev)
    if n > 0 and k > 0:
        rc = _lib.load().tf_quantize_int4(
            w.data_ptr(), n, k, group_size, packed.data_ptr(), scales.data_ptr(), zeros.data_ptr(),
            _lib.dtype_code(dtype), _lib.stream_ptr(dev))
        _lib.check(rc, "quantize_int4_group")
    out_dev = weight.device
    return packed.to(out_dev), scales.to(out_dev), zeros.to(out_dev), k_pad


def unpack_int4(packed: torch.Tensor, k: int | None = None) -> torch.Tensor:
    """Expand K-major packed nibbles [K_pad/2, N] to uint8 codes [K_pad, N] (quant.py:66-74)."""
    if packed.ndim != 2:
        raise ValueError("packed must be 2-D")
    half, n = packed.shape
    dev = _cuda_device(packed)
    p = packed.to(dev).contiguous()
    out = torch.empty((half * 2, n), device=dev, dtype=torch.uint8)
    if half > 0 and n > 0:
        rc = _lib.load().tf_unpack_int4(p.data_ptr(), out.data_ptr(), half * 2, n, _lib.stream_ptr(dev))
        _lib.check(rc, "unpack_int4")
    out = out.to(packed.device)
    return out if k is None else out[:k]


def dequantize_int4(
    packed: torch.Tensor,
    scales: torch.Tensor,
    zeros: torch.Tensor,
    group_size: int = 128,
    dtype: torch.dtype = torch.float16,
) -> torch.Tensor:
    """Reconstruct the dense, K-major weight [K_pad, N] (quant.py:90-105)."""
    half, n = packed.shape
    k_pad = half * 2
    if k_pad % group_size != 0:
        raise ValueError(f"K_pad={k_pad} must be a multiple of group_size={group_size}")
    groups = k_pad // group_size
    for param in (scales, zeros):
        if param.shape != (groups, n):
            got = tuple(param.shape)
            raise ValueError(f"expected group params [G, N] = [{groups}, {n}], got {got}")
    if dtype not in (torch.float16, torch.bfloat16, torch.float32):
        raise ValueError(f"unsupported output dtype {dtype}")
    dev = _cuda_device(packed)
    p = packed.to(dev).contiguous()
    s = scales.to(dev).contiguous()
    z = zeros.to(device=dev, dtype=s.dtype).contiguous()
    if s.dtype not in (torch.float16, torch.bfloat16, torch.float32):
        s, z = s.float(), z.float()
    out = torch.empty((k_pad, n), dtype=dtype, device=dev)
    if k_pad > 0 and n > 0:
        rc = _lib.load().tf_dequantize_int4(
            p.data_ptr(), s.data_ptr(), z.data_ptr(), _lib.dtype_code(s.dtype), out.data_ptr(),
            _lib.dtype_code(dtype), k_pad, n, group_size, _lib.stream_ptr(dev))
        _lib.check(rc, "dequantize_int4")
    return out.to(packed.device)


def quantize_dequantize(
    weight: torch.Tensor,
    group_size: int = 128,
    dtype: torch.dtype = torch.float16,
) -> torch.Tensor:
    """Reference quant.py:108-115: round-trip back to the [N, K] layout."""
    packed, scales, zeros, _ = quantize_int4_group(weight, group_size, dtype)
    dense = dequantize_int4(packed, scales, zeros, group_size, dtype)
    return dense[: weight.shape[1]].t().contiguous()


def quantization_error(weight: torch.Tensor, reconstructed: torch.Tensor) -> dict[str, float]:
    """Reference quant.py:118-127 (error summary of a round trip)."""
    a = weight.detach().to(torch.float32)
    b = reconstructed.detach().to(device=a.device, dtype=torch.float32).reshape_as(a)
    abs_err = (a - b).abs()
    rel = (abs_err / a.abs().clamp_min(1e-3)).mean()
    return {
        "max_abs": abs_err.max().item(),
        "mean_abs": abs_err.mean().item(),
        "mean_rel": rel.item(),
    }
