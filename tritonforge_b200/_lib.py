"""Loader for the native library ``libtritonforge_b200.so`` (C ABI in
``include/tritonforge_b200.h``) and the glue the Python API shares: dtype codes,
status checking, per-device workspaces and the current CUDA stream.

There is no CPU fallback: every op runs the CUDA kernels in this library, and
importing an op without the built library raises immediately.
"""

from __future__ import annotations

import ctypes
import os
import pathlib
import threading

import torch

LIB_PATH = pathlib.Path(__file__).resolve().parent / "libtritonforge_b200.so"

# tf_dtype
F16, BF16, F32, U8 = 0, 1, 2, 3
# tf_regime
REGIME_AUTO, REGIME_GEMV, REGIME_GEMM, REGIME_SIMT = 0, 1, 2, 3
REGIMES = {"auto": REGIME_AUTO, "gemv": REGIME_GEMV, "gemm": REGIME_GEMM, "simt": REGIME_SIMT}

# tf_status
OK = 0
ERR_BAD_SHAPE, ERR_BAD_DTYPE, ERR_UNALIGNED, ERR_CUDA, ERR_TIMEOUT = 1, 2, 3, 4, 5
ERR_WORKSPACE, ERR_BAD_ARG, ERR_UNSUPPORTED = 6, 7, 8

_DT = {torch.float16: F16, torch.bfloat16: BF16, torch.float32: F32, torch.uint8: U8}

_vp, _i64, _i32, _sz, _f32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_size_t, ctypes.c_float

# name -> (restype, argtypes); mirrors include/tritonforge_b200.h
SIGNATURES = {
    "tf_abi_version": (_i32, []),
    "tf_status_string": (ctypes.c_char_p, [_i32]),
    "tf_last_error_message": (ctypes.c_char_p, []),
    "tf_qlinear_workspace_bytes": (_sz, [_i64, _i64, _i64, _i32]),
    "tf_qlinear_gemm_stream_k_grid": (_i32, [_i64, _i64, _i64]),
    "tf_rope_kv_prefill": (_i32, [_vp, _i64, _vp, _i64, _vp, _vp, _vp, _vp, _i64, _i32, _i32, _i32, _i64, _i32,
                                  _vp]),
    "tf_swiglu_gu": (_i32, [_vp, _i64, _vp, _i64, _i64, _i64, _i32, _vp]),
    "tf_qlinear": (_i32, [_vp, _i64, _i32, _vp, _vp, _vp, _i32, _vp, _i32, _vp, _i64,
                          _i64, _i64, _i64, _i64, _i32, _vp, _sz, _vp]),
    "tf_qlinear_ex": (_i32, [_vp, _i64, _i32, _vp, _vp, _vp, _i32, _vp, _i32, _vp, _i64,
                             _i64, _i64, _i64, _i64, _i32, _vp, _sz, _i32, _vp]),
    "tf_qlinear_noalloc": (_i32, [_vp, _i64, _i32, _vp, _vp, _vp, _i32, _vp, _i32, _vp, _i64,
                                  _i64, _i64, _i64, _i64, _i32, _vp]),
    "tf_qlinear_noalloc_error": (_i32, [ctypes.POINTER(ctypes.c_int), _i32, _vp]),
    "tf_workspace_error": (_i32, [_vp, ctypes.POINTER(ctypes.c_int), _vp]),
    "tf_rmsnorm_residual": (_i32, [_vp, _vp, _vp, _i32, _vp, _vp, _i64, _i64, _f32, _i32, _vp]),
    "tf_swiglu": (_i32, [_vp, _vp, _vp, _i64, _i32, _vp]),
    "tf_quantize_int4": (_i32, [_vp, _i64, _i64, _i32, _vp, _vp, _vp, _i32, _vp]),
    "tf_dequantize_int4": (_i32, [_vp, _vp, _vp, _i32, _vp, _i32, _i64, _i64, _i32, _vp]),
    "tf_unpack_int4": (_i32, [_vp, _vp, _i64, _i64, _vp]),
    "tf_rope_kv_append": (_i32, [_vp, _i64, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i32, _i32, _i32, _i64, _i32,
                                 _vp]),
    "tf_decode_attention": (_i32, [_vp, _vp, _vp, _vp, _vp, _i64, _i32, _i32, _i32, _i64, _f32, _i32, _vp]),
    "tf_decode_attention_rope": (_i32, [_vp, _i64, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i32, _i32, _i32, _i64, _f32,
                                        _i32, _vp]),
    "tf_swiglu_strided": (_i32, [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i32, _vp]),
    "tf_qlinear_swiglu": (_i32, [_vp, _i64, _i32, _vp, _vp, _vp, _i32, _vp, _i64, _i64, _i64, _i64, _i64, _i32,
                                 _vp, _sz, _vp]),
    "tf_int4_cm_bytes": (_sz, [_i64, _i64]),
    "tf_repack_int4_cm": (_i32, [_vp, _vp, _i64, _i64, _vp]),
    "tf_qlinear_cm_workspace_bytes": (_sz, [_i64, _i64, _i64]),
    "tf_qlinear_cm": (_i32, [_vp, _i64, _i32, _vp, _vp, _vp, _i32, _vp, _i32, _vp, _i64,
                             _i64, _i64, _i64, _i64, _i32, _vp, _sz, _vp]),
    "tf_qlinear_cm_swiglu": (_i32, [_vp, _i64, _i32, _vp, _vp, _vp, _i32, _vp, _i64, _i64, _i64, _i64, _i64, _i32,
                                    _vp, _sz, _vp]),
    "tf_allreduce_rmsnorm_residual": (_i32, [_vp, _vp, _i64, _i32, _i32, _i32, _vp, _vp, _vp, _i32, _vp, _vp,
                                             _i64, _i64, _f32, _i32, _i32, _vp, _vp]),
    "tf_qlinear_partial": (_i32, [_vp, _i64, _i32, _vp, _vp, _vp, _i32, _vp, _i64, _i64, _i64, _i64, _i64, _i32,
                                  _vp, _sz, _vp]),
    "tf_qlinear_cm_partial": (_i32, [_vp, _i64, _i32, _vp, _vp, _vp, _i32, _vp, _i64, _i64, _i64, _i64, _i64, _i32,
                                     _vp, _sz, _vp]),
    "tf_embed_gather": (_i32, [_vp, _i64, _vp, _vp, _i64, _vp, _i64, _i64, _i64, _i64, _i32, _vp]),
    "tf_lm_head_workspace_bytes": (_sz, [_i64]),
    "tf_lm_head_argmax": (_i32, [_vp, _i64, _vp, _i64, _i64, _i64, _i64, _i32, _vp, _i64, _vp, _vp, _i64, _vp, _i32,
                                 _vp, _sz, _vp]),
    "tf_best_of_ranks": (_i32, [_vp, _vp, _i32, _i64, _vp]),
}

_lib: ctypes.CDLL | None = None
_lock = threading.Lock()


def load() -> ctypes.CDLL:
    """Load the native library (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            path = os.environ.get("TRITONFORGE_B200_LIB", str(LIB_PATH))
            if not pathlib.Path(path).exists():
                raise RuntimeError(
                    f"tritonforge_b200 native library not found at {path}; build it with "
                    "`make -C tritonforge_b200/csrc` (or __graft_entry__.build())")
            lib = ctypes.CDLL(path)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DT[dt]
    except KeyError:
        raise ValueError(f"unsupported dtype {dt}") from None


def check(rc: int, what: str) -> None:
    if rc != OK:
        lib = load()
        msg = lib.tf_last_error_message().decode(errors="replace")
        status = lib.tf_status_string(rc).decode()
        raise RuntimeError(f"{what} failed: {status} ({rc}): {msg}")


def require_cuda(*tensors: torch.Tensor | None) -> torch.device:
    """All given tensors must live on one CUDA device; returns it."""
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError(
                "tritonforge_b200 ops run on CUDA only (got a tensor on "
                f"{t.device}); there is no CPU implementation")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError(f"tensors on different devices: {dev} vs {t.device}")
    if dev is None:
        raise RuntimeError("no CUDA tensor given")
    return dev


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


class _Workspaces:
    """Zero-initialised scratch handed to the kernels, one buffer per (device,
    stream). Its 256-byte header is shared by every kernel: word 0 is the device
    error word of their bounded waits (a wait that gives up after 1 s sets a
    bit there and the launch still reports success). After the header,
    tf_lm_head_argmax keeps a counter it leaves zeroed and per-CTA partial
    results, and the prefill GEMM's stream-K schedule keeps partial tiles
    (from byte 512) and arrival counters it leaves zeroed (the buffer's last
    64 KiB); a buffer smaller than tf_qlinear_workspace_bytes runs the GEMM
    one tile per CTA instead. Calls that share a buffer are ordered on their
    stream. ``errors`` reads the word of every buffer.

    A buffer is zeroed only when it is (re)allocated. Reallocation happens
    outside any CUDA-graph capture: callers that capture size it first with
    ``reserve`` (or run the captured work once on the capture stream).
    """

    def __init__(self) -> None:
        self._bufs: dict[tuple[int, int], torch.Tensor] = {}

    def get(self, device: torch.device, nbytes: int) -> torch.Tensor:
        idx = device.index if device.index is not None else torch.cuda.current_device()
        key = (idx, torch.cuda.current_stream(idx).cuda_stream)
        buf = self._bufs.get(key)
        if buf is None or buf.numel() < nbytes:
            size = max(nbytes, 1 << 20, 0 if buf is None else 2 * buf.numel())
            buf = torch.zeros(size, dtype=torch.uint8, device=torch.device("cuda", idx))
            self._bufs[key] = buf
        return buf

    def reserve(self, device: torch.device, nbytes: int) -> None:
        self.get(device, nbytes)

    def errors(self, device: torch.device | None = None, clear: bool = False) -> int:
        """OR of the error words of this process's workspaces (on `device`, or
        all devices): 0 when every kernel that used them completed its bounded
        waits. Synchronises the devices involved; `clear` zeroes the words."""
        bits = 0
        for (idx, _), buf in list(self._bufs.items()):
            if device is not None and device.index is not None and idx != device.index:
                continue
            torch.cuda.synchronize(idx)
            word = buf[:4].view(torch.int32)
            bits |= int(word.item())
            if clear:
                word.zero_()
        return bits


workspaces = _Workspaces()
