"""Tensor-parallel decode checks shared by the GPU tests.

`ThreadReducer` emulates TP ranks as threads on one GPU (host barrier, the
fp32 partials summed on the device in rank order, as the fused all-reduce
does); run as a script under
torchrun this module is the NCCL worker: every rank builds the same full
weights, decodes its shard with the all-reduce captured in a CUDA graph, and
rank 0 compares the logits with a tp=1 decode of the full weights.
"""

from __future__ import annotations

import json
import os
import sys
import threading

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

from tritonforge_b200.decode import DECODE_MAX_TOL, DECODE_MEAN_TOL, QwenDecoder, QwenWeights  # noqa: E402,F401


class ThreadReducer:
    """In-place sum across `n` threads of one process (one thread per rank)."""

    def __init__(self, n: int, timeout_s: float = 120.0):
        self.n = n
        self.slots: list = [None] * n
        self.bar = threading.Barrier(n, timeout=timeout_s)

    def member(self, rank: int) -> "_Member":
        return _Member(self, rank)


class _Member:
    def __init__(self, red: ThreadReducer, rank: int):
        self.red, self.rank = red, rank

    def all_reduce(self, t: torch.Tensor) -> None:
        red = self.red
        torch.cuda.current_stream(t.device).synchronize()
        red.slots[self.rank] = t
        red.bar.wait()
        if self.rank == 0:
            acc = red.slots[0].clone()
            for other in red.slots[1:]:
                acc.add_(other)
            for s in red.slots:
                s.copy_(acc)
            torch.cuda.current_stream(t.device).synchronize()
        red.bar.wait()


def copy_cache(src: QwenDecoder, dst: QwenDecoder, tp: int, rank: int) -> None:
    """Give a TP rank the kv heads of `src`'s cache that it owns, and src's tokens/position."""
    h = dst.Hkv
    dst.k_cache.copy_(src.k_cache[:, :, rank * h:(rank + 1) * h])
    dst.v_cache.copy_(src.v_cache[:, :, rank * h:(rank + 1) * h])
    dst.tokens.copy_(src.tokens)
    dst.pos.copy_(src.pos)


def excess_error(got: torch.Tensor, want: torch.Tensor, ulps: int = 1) -> tuple[float, float]:
    """(max(|got - want| - ulps x bf16 ulp(want)), RMS(want)): the difference
    that the outputs' own final roundings (`ulps` of them after the value the
    two computations sum in different fp32 orders) do not explain."""
    w = want.float()
    ulp = torch.ldexp(torch.ones_like(w), torch.frexp(w)[1] - 8)
    err = float(((got.float() - w).abs() - ulps * ulp).clamp_min(0).max())
    return err, float(w.pow(2).mean().sqrt())


# DECODE_MAX_TOL / DECODE_MEAN_TOL (from the decoder): the model-level bounds
# between two decodes of the same bf16 weights whose only difference is the fp32
# summation order (see logits_close).


def logits_close(got: torch.Tensor, ref: torch.Tensor, tol: float = DECODE_MAX_TOL,
                 mean_tol: float = DECODE_MEAN_TOL) -> tuple[bool, float, float]:
    """Logits of one whole decode against another decode of the same weights
    (a tensor-parallel one against tp=1, or another weight layout): max(|got -
    ref| - ulp(ref)) <= tol x RMS(ref) and mean |got - ref| <= mean_tol x RMS.
    Returns (ok, that max, RMS).

    Every op of both decodes meets the per-kernel contract (2e-2 x RMS against
    the oracle on identical inputs, tested op by op, including the sharded
    row-parallel reduction in tp_parity / test_tp_row_parallel_op). Between
    two whole decodes the inputs of each op already differ: the fp32
    summation order (split-K partitions, the cross-rank sum, attention chunks)
    moves a rounded bf16 value by one ulp now and then, and those flips feed
    every later op. Measured noise floor of that effect with no tensor
    parallelism at all: two single-GPU decodes of 2-layer 7B-shaped weights
    that differ only in the GEMV kernel (K-major mma.sync vs column-major
    tcgen05) differ by 2.9-4.7% of the logit RMS (max beyond one ulp, over
    2.4-7.3M logits; mean up to 0.58%), and a host restatement with fp32
    against fp64 accumulation at identical rounding points, without attention,
    by 1.9% (mean 0.15%). One ulp of each logit is its own rounding (near
    5 x RMS a bf16 ulp is ~2.6% of the RMS); the bounds on top of it, 6e-2 for
    the max and 1e-2 for the mean, are that floor with headroom. A wrong
    column, row or scale moves logits by a sizeable fraction of the RMS.
    Returns (ok, max beyond one ulp, RMS, mean)."""
    ref32 = ref.float()
    ulp = torch.ldexp(torch.ones_like(ref32), torch.frexp(ref32)[1] - 8)  # bf16 ulp of each reference logit
    diff = (got.float() - ref32).abs()
    err = float((diff - ulp).clamp_min(0).max())
    rms = float(ref32.pow(2).mean().sqrt())
    mean = float(diff.mean())
    return err <= tol * rms and mean <= mean_tol * rms, err, rms, mean


def near_tie(ref_logits: torch.Tensor, ref_tok: torch.Tensor, got_tok: torch.Tensor, rms: float,
             tol: float = 2e-2) -> tuple[bool, float]:
    """Rows whose greedy tokens differ must be genuine near-ties of the
    reference: the reference scores the other token within tol x RMS of its
    own choice. Returns (whether all differing rows are such ties, the largest
    reference gap among them)."""
    ref32 = ref_logits.float()
    rows = (got_tok != ref_tok).nonzero().flatten()
    if rows.numel() == 0:
        return True, 0.0
    gap = float((ref32[rows, ref_tok[rows]] - ref32[rows, got_tok[rows]]).max())
    return gap <= tol * rms, gap


def _nccl_main() -> int:
    import datetime

    import torch.distributed as dist

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    name = os.environ.get("TP_CHECK_MODEL", "7b")
    layers = int(os.environ.get("TP_CHECK_LAYERS", "2"))
    steps = int(os.environ.get("TP_CHECK_STEPS", "4"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    B, T = int(os.environ.get("TP_CHECK_BATCH", "4")), 96  # 9..128: the column-major tcgen05 decode kernel
    full = QwenWeights.synthetic(name, tp=1, rank=0, dtype=torch.bfloat16, device=dev, seed=3, layers=layers)
    ref = QwenDecoder(full, B, T)
    ref.fill_cache(40, seed=5)  # same seed on every rank -> same cache everywhere
    fused = os.environ.get("TP_CHECK_FUSED", "1") == "1"  # fused all-reduce + RMSNorm, or NCCL
    dec = QwenDecoder(full.shard(world, rank), B, T, group=dist.group.WORLD, fused_allreduce=fused)
    copy_cache(ref, dec, world, rank)
    report = {"rank": rank, "ok": True, "steps": []}
    dec.capture()
    v0, nv = dec.v0, dec.lm_head.shape[0]  # this rank's vocabulary slice (vocab-parallel lm_head)
    same_all = True
    for i in range(steps):
        ref.step()
        dec.graph.replay()
        ok, err, rms, mean = logits_close(dec.buf["logits"], ref.buf["logits"][:, v0:v0 + nv])
        same_tok = bool(torch.equal(dec.tokens, ref.tokens))
        tie_ok, gap = near_tie(ref.buf["logits"], ref.tokens, dec.tokens, rms)
        ok &= tie_ok
        report["steps"].append({"err": err, "mean": mean, "rms": rms, "tokens_equal": same_tok, "tie_gap": gap})
        report["ok"] &= ok
        # ranks must agree on the tokens bit for bit
        gathered = [torch.empty_like(dec.tokens) for _ in range(world)]
        dist.all_gather(gathered, dec.tokens)
        same_all &= all(torch.equal(gathered[0], g) for g in gathered)
        dec.tokens.copy_(ref.tokens)  # keep the two decodes on the same tokens
    report["ranks_identical"] = same_all
    report["fused_allreduce"] = dec.fused_allreduce
    report["device_errors"] = dec.device_errors() | ref.device_errors()
    report["ok"] &= report["device_errors"] == 0
    report["ok"] &= report["ranks_identical"]
    torch.cuda.synchronize()
    dec.release()
    dist.barrier()
    dist.destroy_process_group()
    if rank == 0:
        print("TP_CHECK " + json.dumps(report), flush=True)
    return 0 if report["ok"] else 1


if __name__ == "__main__":
    sys.exit(_nccl_main())
