"""GPU tests of tf_allreduce_rmsnorm_residual on one GPU.

The peers of rank 0 are emulated by buffers on the same GPU whose signal-pad
slots the test sets before each call (no second kernel waits on this one):
the result must equal the oracle's rmsnorm_residual of round(sum of the
partials in rank order) and the residual, the kernel must signal every peer's
pad, and the call count must advance. A peer that never signals makes the
bounded wait give up after ~1 s with error bit 16 (no GPU fault, the context
stays usable)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import ops as oops
from oracle import quant as oquant
from tests.parity import NP_DT, assert_rms_close, f32
from tritonforge_b200 import _lib

pytestmark = pytest.mark.gpu

SLOT = 64


def _make(world, m, n, dtype, seed, part_dtype=None):
    g = torch.Generator(device="cuda").manual_seed(seed)
    parts = [(torch.randn(m, n, device="cuda", generator=g) * 0.5).to(part_dtype or dtype) for _ in range(world)]
    pads = [torch.zeros(SLOT + 8, dtype=torch.int32, device="cuda") for _ in range(world)]
    res = torch.randn(m, n, device="cuda", generator=g).to(dtype)
    w = (1 + 0.02 * torch.randn(n, device="cuda", generator=g)).to(dtype)
    bufs = torch.tensor([p.data_ptr() for p in parts], dtype=torch.int64, device="cuda")
    pad_ptrs = torch.tensor([p.data_ptr() for p in pads], dtype=torch.int64, device="cuda")
    return parts, pads, res, w, bufs, pad_ptrs


def _call(bufs, pad_ptrs, world, ctr, res, w, normed, summed, err, dtype, part_dtype=None):
    m, n = res.shape
    rc = _lib.load().tf_allreduce_rmsnorm_residual(
        bufs.data_ptr(), pad_ptrs.data_ptr(), 0, SLOT, 0, world, ctr.data_ptr(), res.data_ptr(), w.data_ptr(),
        _lib.dtype_code(w.dtype), normed.data_ptr(), summed.data_ptr(), m, n, 1e-6, _lib.dtype_code(dtype),
        _lib.dtype_code(part_dtype or dtype), err.data_ptr(), _lib.stream_ptr(res.device))
    _lib.check(rc, "allreduce_rmsnorm_residual")


@pytest.mark.parametrize("partials", ["fp32", "model"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("world,m,n", [(1, 4, 896), (2, 32, 8192), (4, 8, 3584), (8, 3, 8192)])
def test_fused_allreduce_rmsnorm(world, m, n, dtype, partials):
    """fp32 partials (tf_qlinear_partial's unrounded sums, what the decoder
    hands over) and partials already rounded to the model dtype."""
    pdt = torch.float32 if partials == "fp32" else dtype
    parts, pads, res, w, bufs, pad_ptrs = _make(world, m, n, dtype, seed=world * 10 + m, part_dtype=pdt)
    ctr = torch.zeros(2, dtype=torch.int32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    normed = torch.empty_like(res)
    summed = torch.empty_like(res)
    dt = NP_DT[dtype]
    for call in (1, 2, 3):
        for p in range(1, world):
            pads[0][SLOT + p] = call  # peer p has signalled this call
        _call(bufs, pad_ptrs, world, ctr, res, w, normed, summed, err, dtype, pdt)
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        assert int(ctr[0].item()) == call and int(ctr[1].item()) == 0
        for p in range(world):
            assert int(pads[p][SLOT].item()) == call, "rank 0 signals every rank's pad once per call"
        acc = np.zeros((m, n), np.float32)
        for p in parts:  # fp32 sum in rank order, rounded once to the model dtype
            acc = acc + f32(p)
        o = oquant.round_to(acc, dt)
        ref_n, ref_s = oops.rmsnorm_residual(o, f32(res), f32(w), 1e-6, dt)
        assert torch.equal(summed.cpu().float(), torch.from_numpy(np.asarray(ref_s, np.float32)))
        assert_rms_close(normed, ref_n, dtype, "fused all-reduce rmsnorm", max_mismatch=0.01)


def test_fused_allreduce_missing_peer_times_out():
    parts, pads, res, w, bufs, pad_ptrs = _make(2, 2, 1024, torch.bfloat16, seed=5)
    ctr = torch.zeros(2, dtype=torch.int32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    normed = torch.zeros_like(res)
    summed = torch.zeros_like(res)
    _call(bufs, pad_ptrs, 2, ctr, res, w, normed, summed, err, torch.bfloat16)  # peer 1 never signals
    torch.cuda.synchronize()
    assert int(err.item()) & 16
    assert int(ctr[0].item()) == 1  # the call still completes and counts
    assert normed.abs().sum().item() == 0 and summed.abs().sum().item() == 0  # nothing written
    # the context is still usable
    x = torch.ones(4, device="cuda")
    assert float((x * 2).sum().item()) == 8.0
