"""CPU tests of the tensor-parallel host logic (gloo ranks, no GPU): shard
sizes, quantise-then-shard == shard-then-quantise (bit-exact, oracle
quantizer), column/row-parallel equivalence with the unsharded oracle linear
through real collectives, and a rank that leaves before a collective making
the survivor fail cleanly on the host within the process-group timeout."""

from __future__ import annotations

import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import ops as oops
from oracle import quant as oquant
from tritonforge_b200.tp import GROUP, TPLayout, shard_cols, shard_rows, split_even


def test_split_even():
    for total, parts in [(231, 8), (231, 4), (231, 2), (148, 2), (148, 4), (7, 8), (38, 3)]:
        spans = [split_even(total, parts, r) for r in range(parts)]
        assert spans[0][0] == 0 and spans[-1][1] == total
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
        sizes = [e - s for s, e in spans]
        assert max(sizes) - min(sizes) <= 1
    assert [e - s for s, e in (split_even(231, 8, r) for r in range(8))] == [29] * 7 + [28]


@pytest.mark.parametrize("name,tps", [("7b", (1, 2, 4)), ("72b", (1, 2, 4, 8))])
def test_layouts(name, tps):
    from tritonforge_b200.decode import QWEN25

    s = QWEN25[name]
    for tp in tps:
        widths = []
        for r in range(tp):
            lay = TPLayout(tp, r, s.hidden, s.inter, s.heads, s.kv_heads, s.head_dim)
            c0, c1 = lay.inter_cols
            assert c0 % GROUP == 0 and c1 % GROUP == 0
            widths.append(c1 - c0)
            assert lay.q_heads * tp == s.heads and lay.kv_local * tp == s.kv_heads
        assert sum(widths) == s.inter
    with pytest.raises(ValueError):
        TPLayout(8, 0, s.hidden, s.inter, s.heads, 4 if name == "7b" else 12, s.head_dim)


def test_quantize_then_shard_is_bit_exact():
    rng = np.random.default_rng(0)
    w = (rng.standard_normal((96, 640)) * 0.02).astype(np.float32)  # [N, K], K = 5 groups
    packed, scales, zeros, _ = oquant.quantize_int4_group(w, GROUP)
    t = [torch.from_numpy(a) for a in (packed, scales, zeros)]
    # row shard of groups 1..3 == quantising only those input columns
    p, s, z = shard_rows(*t, 128, 512)
    p2, s2, z2, _ = oquant.quantize_int4_group(w[:, 128:512], GROUP)
    assert np.array_equal(p.numpy(), p2) and np.array_equal(s.numpy(), s2) and np.array_equal(z.numpy(), z2)
    # column shard == quantising only those output rows of W
    p, s, z, _ = shard_cols(*t, None, 32, 80)
    p2, s2, z2, _ = oquant.quantize_int4_group(w[32:80], GROUP)
    assert np.array_equal(p.numpy(), p2) and np.array_equal(s.numpy(), s2) and np.array_equal(z.numpy(), z2)
    with pytest.raises(ValueError):
        shard_rows(*t, 64, 512)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=60):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))


def _equivalence_worker(rank, world, port, q):
    try:
        _init(rank, world, port)
        rng = np.random.default_rng(7)
        hidden, inter = 256, 3 * GROUP * world - GROUP  # uneven intermediate split
        x = rng.standard_normal((4, hidden)).astype(np.float16).astype(np.float32)
        w_up = (rng.standard_normal((inter, hidden)) * 0.02).astype(np.float32)    # column-parallel
        w_down = (rng.standard_normal((hidden, inter)) * 0.02).astype(np.float32)  # row-parallel
        pu, su, zu, _ = oquant.quantize_int4_group(w_up, GROUP)
        pd, sd, zd, _ = oquant.quantize_int4_group(w_down, GROUP)
        f16 = lambda b: oquant.half_bits_to_f32(b, "float16")  # noqa: E731
        full_up = oops.quantized_linear(x, pu, f16(su), f16(zu), None, GROUP)
        g0, g1 = split_even(inter // GROUP, world, rank)
        c0, c1 = g0 * GROUP, g1 * GROUP
        t = lambda a: torch.from_numpy(np.ascontiguousarray(a))  # noqa: E731
        p, s, z, _ = shard_cols(t(pu), t(su), t(zu), None, c0, c1)
        local_up = oops.quantized_linear(x, p.numpy(), f16(s.numpy()), f16(z.numpy()), None, GROUP)
        # column-parallel: the local columns equal the unsharded ones exactly
        ok_cols = np.array_equal(local_up, full_up[:, c0:c1])
        # row-parallel: fp32 partial sums over the local groups, added by an all-reduce
        p, s, z = shard_rows(t(pd), t(sd), t(zd), c0, c1)
        wloc = oquant.round_to(oquant.dequantize_int4_f32(p.numpy(), f16(s.numpy()), f16(z.numpy()), GROUP),
                               "float16")
        part = torch.from_numpy((full_up[:, c0:c1].astype(np.float64) @ wloc.astype(np.float64)).astype(np.float32))
        dist.all_reduce(part)
        wfull = oquant.round_to(oquant.dequantize_int4_f32(pd, f16(sd), f16(zd), GROUP), "float16")
        ref = (full_up.astype(np.float64) @ wfull.astype(np.float64)).astype(np.float32)
        err = float(np.max(np.abs(part.numpy() - ref)))
        q.put((rank, ok_cols, err, c1 - c0))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, False, repr(e), 0))


@pytest.mark.parametrize("world", [2, 4])
def test_tp_equivalence_gloo(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_equivalence_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    widths = []
    for rank, ok_cols, err, width in results:
        assert ok_cols is True, (rank, err)
        assert isinstance(err, float) and err < 1e-4, (rank, err)
        widths.append(width)
    assert sum(widths) == 3 * GROUP * world - GROUP and len(set(widths)) == 2  # uneven split exercised


def _fault_worker(rank, world, port, q):
    _init(rank, world, port, timeout_s=5)
    t = torch.ones(4)
    if rank == 1:
        os._exit(0)  # leaves between steps, before the collective
    try:
        dist.all_reduce(t)
        q.put((rank, "completed"))
    except Exception as e:
        q.put((rank, f"failed: {type(e).__name__}"))


def test_rank_exit_fails_cleanly_on_host():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_fault_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    rank, status = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert rank == 0 and status.startswith("failed"), status


def _argmax_worker(rank, world, port, q):
    try:
        _init(rank, world, port)
        from tritonforge_b200.tp import best_of_ranks, local_best

        g = torch.Generator().manual_seed(11)
        vocab, b = 1001, 6
        logits = torch.randint(-4, 5, (b, vocab), generator=g).to(torch.bfloat16)  # many ties
        logits[0, 3] = 9.0
        logits[0, 700] = 9.0   # tie across ranks: the smaller id must win
        logits[1, :] = 0.0     # all equal: id 0
        v0, v1 = split_even(vocab, world, rank)
        best = torch.empty(b, 2)
        arg = torch.empty(b, dtype=torch.long)
        local_best(logits[:, v0:v1].contiguous(), v0, best, arg)
        all_best = torch.empty(world, b, 2)
        dist.all_gather_into_tensor(all_best.view(-1, 2), best)
        tok = best_of_ranks(all_best).long()
        q.put((rank, bool(torch.equal(tok, torch.argmax(logits, dim=-1))), tok.tolist()))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, False, repr(e)))


@pytest.mark.parametrize("world", [2, 3])
def test_vocab_parallel_argmax_gloo(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_argmax_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, ok, info in results:
        assert ok, (rank, info)


def test_near_tie_check():
    """The TP token check accepts a differing greedy token only where the
    reference scores it within the contract's 2e-2 x RMS of its own choice."""
    import torch

    from tests.tp_check import logits_close, near_tie

    ref = torch.tensor([[1.00, 0.99, 0.0], [2.0, 1.0, 0.5]])
    ref_tok = torch.tensor([0, 0])
    ok, gap = near_tie(ref, ref_tok, torch.tensor([1, 0]), rms=1.0)
    assert ok and abs(gap - 0.01) < 1e-6
    ok, gap = near_tie(ref, ref_tok, torch.tensor([0, 1]), rms=1.0)
    assert not ok and abs(gap - 1.0) < 1e-6
    assert near_tie(ref, ref_tok, ref_tok, rms=1.0) == (True, 0.0)
    # logits: max beyond one ulp against 6e-2 x RMS, mean against 2e-3 x RMS
    base = torch.randn(4, 1000, generator=torch.Generator().manual_seed(0))
    rms = float(base.pow(2).mean().sqrt())
    bumped = base.clone()
    bumped[0, 0] += 0.05 * rms
    assert logits_close(bumped, base)[0]
    bumped[0, 1] += 0.12 * rms  # beyond one bf16 ulp of any value here plus the 6e-2 x RMS bound
    assert not logits_close(bumped, base)[0]
