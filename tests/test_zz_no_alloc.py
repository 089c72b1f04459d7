"""GPU test of tf_qlinear_noalloc, the int4 linear for callers that cannot
allocate device memory (a plugin inside a framework whose allocator owns all
device memory, a host runtime behind an FFI with no CUDA allocator): it takes
its scratch from an array built into the library instead of a workspace.

It is called here through the C ABI and its output is compared with the
regular entry point's (tf_qlinear through kernels.quantized_linear) and with
the oracle, on two calls in a row, with the parity tolerance of the other
tests; after the calls the array's error word (tf_qlinear_noalloc_error) must
be 0, i.e. every bounded device wait of those calls completed. This file is
collected last so that a run stopping at the first failure has run everything
else first; it also passes when run alone in a fresh process (the first call
sets the array up).
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from tests.parity import assert_rms_close, oracle_linear
from tritonforge_b200 import _lib, kernels, quant

pytestmark = pytest.mark.gpu


def _noalloc(x, packed, scales, zeros, bias, out, group=128):
    lib = _lib.load()
    rc = lib.tf_qlinear_noalloc(
        x.data_ptr(), x.stride(0), _lib.dtype_code(x.dtype), packed.data_ptr(), scales.data_ptr(),
        zeros.data_ptr(), _lib.dtype_code(scales.dtype), _lib.ptr(bias),
        _lib.dtype_code(bias.dtype) if bias is not None else 0, out.data_ptr(), out.stride(0),
        x.shape[0], packed.shape[1], x.shape[1], packed.shape[0] * 2, group, _lib.stream_ptr(x.device))
    _lib.check(rc, "tf_qlinear_noalloc")
    return out


@pytest.mark.parametrize("m,n,k,dtype", [
    (1, 4864, 896, torch.float16),      # decode GEMV, 0.5B gate/up
    (8, 18944, 3584, torch.bfloat16),   # decode GEMV, 7B gate/up (cluster split-K)
    (16, 896, 4864, torch.float16),     # decode GEMV, 0.5B down
    (5, 127, 129, torch.float16),       # generic kernel (ragged N, odd K)
    (40, 512, 256, torch.bfloat16),     # generic kernel (M > 32)
])
def test_noalloc_matches_regular_entry_point(m, n, k, dtype):
    g = torch.Generator().manual_seed(m * 31 + n)
    x = torch.randn(m, k, generator=g).to(dtype).cuda()
    w = (torch.randn(n, k, generator=g) * 0.02).cuda()
    packed, scales, zeros, _ = quant.quantize_int4_group(w, 128, dtype)
    bias = torch.randn(n, generator=g).to(dtype).cuda()
    want = kernels.quantized_linear(x, packed, scales, zeros, bias)
    ref = oracle_linear(x, packed, scales, zeros, bias)
    for _ in range(2):  # the shared scratch keeps the previous call's contents
        out = torch.full((m, n), float("nan"), dtype=dtype, device="cuda")
        got = _noalloc(x, packed, scales, zeros, bias, out)
        torch.cuda.synchronize()
        assert_rms_close(got, want.float().cpu().numpy(), dtype, f"noalloc {m}x{n}x{k} vs tf_qlinear")
        assert_rms_close(got, ref, dtype, f"noalloc {m}x{n}x{k} vs oracle")
    word = ctypes.c_int(-1)
    rc = _lib.load().tf_qlinear_noalloc_error(ctypes.byref(word), 1, _lib.stream_ptr(x.device))
    assert rc == _lib.OK and word.value == 0, (rc, word.value)
