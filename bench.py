"""Decode benchmark: Qwen2.5-shaped int4 models on the B200 kernels.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--model 72b|7b|0.5b] [--batch B] [--prompt T]

Default workload: the Qwen2.5-72B architecture (80 layers, hidden 8192, 64 q /
8 kv heads of 128, intermediate 29568, vocab 152064), random-init int4
group-128 weights (bf16 scales, zeros and activations), batch 32, a KV cache of
4096 prompt positions filled with random values, greedy decode. The model is
tensor-parallel over the N ranks (column-parallel q/k/v/gate/up, row-parallel
o/down with an NCCL all-reduce after each, captured in the step's CUDA graph):
total work is fixed as N grows (strong scaling). `--model 7b` is the 7B shape
the same way; `--model 0.5b` is the transformers Qwen2.5-0.5B (fp16) patched
with the int4 QuantLinear, prefilled through the model, one replica per rank.
One step = one decoded token for each of the B sequences (all layers,
lm_head, argmax).

Prints one JSON line. `value` is decode tokens/s of the whole job, timed on
the device (CUDA events, max over ranks) with tokens fed back on the device;
`e2e` is the same metric through the decoder's public step with the step's
input tokens copied from pinned host memory and its output tokens read back
every step. `roofline` is the int4 GEMV (the kernel that streams the
weights): one step's GEMV launches replayed alone in a CUDA graph, algorithmic
bytes / device time against the measured HBM copy bandwidth. `cpu_baseline`
times the reference's CPU path (dequantize-then-matmul int4 projections,
restated in oracle/) on this host's cores: for the 0.5B model whole decode
steps, for 7B/72B one decoder layer plus the lm_head, extrapolated to all
layers.

For 7B/72B the line also carries `prefill`: the time to first token of one
2048-token prompt (`--prefill-len`) through the engine's own prefill (the
tcgen05 int4 GEMM at M = prompt length for every projection), timed before the
decode weights are converted.

`--impl reference` times that same CPU path as the reference arm (rank 0 only).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "int4 GEMV HBM GB/s (% of peak) at decode; Qwen2.5-shape decode tok/s at 1/2/4/8 GPU"


def _peaks() -> dict:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return {"hbm_gbs": float(p["hbm_gbs"]), "source": "measured"}
    except Exception:
        return {"hbm_gbs": 6650.0, "source": "fallback"}


def _peaks_tensor() -> dict:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return {"bf16_tflops": float(json.load(f)["bf16_tflops"]), "source": "measured"}
    except Exception:
        return {"bf16_tflops": 1590.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clock / throttle sampling while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int) -> None:
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []
        self.thread = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            time.sleep(0.3)
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.2)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        loaded = [v for v in sm if mx and v > 0.5 * mx] or sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def _dist():
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not dist.is_initialized():
        import datetime
        if torch.cuda.is_available():
            torch.cuda.set_device(local)
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", local))
        else:
            dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    return world, rank, local


def _max_over_ranks(value: float, world: int) -> float:
    if world == 1:
        return value
    import torch
    import torch.distributed as dist

    t = torch.tensor([value], dtype=torch.float64, device="cuda" if torch.cuda.is_available() else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def build_model(args, device):
    """Random-init model (seeded) on the GPU, patched with int4 QuantLinears;
    also returns an unpatched CPU copy for the CPU baseline when asked."""
    import copy

    import torch

    from tritonforge_b200.decode import random_qwen2
    from tritonforge_b200.integration import patch_model

    model = random_qwen2(args.model, seed=0)
    cpu_copy = copy.deepcopy(model) if args.want_cpu else None
    model = model.to(device)
    patch_model(model, group_size=128, dtype=torch.float16)
    return model, cpu_copy


def prompt_ids(args, vocab: int, rank: int):
    import torch

    g = torch.Generator().manual_seed(1000 + rank)
    return torch.randint(0, vocab, (args.batch, args.prompt), generator=g)


def cpu_decode_rate(cpu_model, prompt, steps: int, budget_s: float) -> tuple[float, int, int, str]:
    """Decode tok/s of the reference's CPU path on this host (bounded sample)."""
    import torch

    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    with torch.no_grad():
        out = cpu_model(prompt, use_cache=True)
        past = out.past_key_values
        nxt = out.logits[:, -1, :].argmax(-1, keepdim=True)
        done, t0 = 0, time.perf_counter()
        while done < steps:
            out = cpu_model(nxt, past_key_values=past, use_cache=True)
            past = out.past_key_values
            nxt = out.logits[:, -1, :].argmax(-1, keepdim=True)
            done += 1
            if time.perf_counter() - t0 > budget_s:
                break
        dt = time.perf_counter() - t0
    b = prompt.shape[0]
    sample = f"{done} decode steps x batch {b} after a {prompt.shape[1]}-token prefill, {dt:.1f} s"
    return b * done / dt, cores, done, sample


def cpu_layer_rate(args, budget_s: float) -> tuple[float, int, str, int]:
    """Decode tok/s of the reference's CPU path for a 7B/72B shape on this
    host, from one decoder layer (timed over a few decode steps after one
    untimed step) plus the final norm, lm_head and argmax, extrapolated to all
    layers. Everything is built on the host (oracle.cpu_decode.CpuLayer.random:
    int4 tensors of the layer's shapes with seeded random contents, whose
    values do not change the CPU path's cost); no GPU code runs.
    Returns (tok/s, cores, sample description, timed layer-steps)."""
    import torch

    from oracle.cpu_decode import CpuLayer
    from tritonforge_b200.decode import QWEN25, hf_config

    shape = QWEN25[args.model]
    dt = torch.bfloat16
    layer = CpuLayer.random(shape.hidden, shape.inter, shape.heads, shape.kv_heads, shape.head_dim, shape.eps, dt,
                            seed=0)
    t_max = args.prompt + 16
    from transformers.models.qwen2.modeling_qwen2 import Qwen2RotaryEmbedding

    rot = Qwen2RotaryEmbedding(hf_config(shape))
    cos, sin = (t[0] for t in rot(torch.zeros(1, 1, 8, dtype=dt), torch.arange(t_max).unsqueeze(0)))
    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    g = torch.Generator().manual_seed(5)
    lm_head = (torch.randn(shape.vocab, shape.hidden, generator=g) * 0.02).to(dt)
    final_norm = torch.ones(shape.hidden, dtype=dt)
    b = args.batch
    x = torch.randn(b, shape.hidden, generator=g).to(dt)
    kc = torch.randn(b, shape.kv_heads, t_max, shape.head_dim, generator=g).to(dt)
    vc = torch.randn(b, shape.kv_heads, t_max, shape.head_dim, generator=g).to(dt)
    layer.step(x, kc, vc, args.prompt, cos, sin)  # untimed warm-up step
    n, t0 = 0, time.perf_counter()
    while True:
        layer.step(x, kc, vc, args.prompt + 1 + n, cos, sin)
        n += 1
        if n >= 8 or time.perf_counter() - t0 > budget_s:
            break
    t_layer = (time.perf_counter() - t0) / n
    t1 = time.perf_counter()
    with torch.no_grad():
        h = x.float()
        h = (final_norm * (h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + shape.eps)).to(x.dtype))
        (h @ lm_head.t()).argmax(-1)
    t_head = time.perf_counter() - t1
    step_s = shape.layers * t_layer + t_head
    sample = (f"1 of {shape.layers} decoder layers (int4 g128, host-built seeded random codes) timed over {n} decode "
              f"steps after 1 untimed (batch {b}, context {args.prompt}) plus final norm/lm_head/argmax "
              f"({t_head:.2f} s), extrapolated to {shape.layers} layers: {step_s:.1f} s per step")
    return b / step_s, cores, sample, n


def run_reference(args) -> None:
    """The reference arm: the reference's CPU path on this host's cores, built
    and run on the host only (no GPU code of this repository is loaded)."""
    if int(os.environ.get("RANK", "0")) != 0:
        return  # rank 0 alone runs the CPU path; the other ranks exit without work
    import torch

    budget = float(os.environ.get("TF_REF_BUDGET_S", "120"))
    if args.model == "0.5b":
        from oracle.cpu_decode import quantize_model_on_cpu
        from tritonforge_b200.decode import random_qwen2

        cpu_model = quantize_model_on_cpu(random_qwen2(args.model, seed=0), 128, torch.float16)
        prompt = prompt_ids(args, cpu_model.config.vocab_size, 0)
        rate, cores, done, sample = cpu_decode_rate(cpu_model, prompt, args.steps, budget)
        warm = 0
        sample = "oracle-quantised on the host; " + sample
    else:
        rate, cores, sample, done = cpu_layer_rate(args, budget)
        warm = 1
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": rate, "unit": "tok/s", "n_gpus": args.gpus,
        "steps": done, "warmup": warm, "ms_per_step": 1000.0 * args.batch / rate, "higher_is_better": True,
        "scaling": "strong" if args.model != "0.5b" else "weak", "vs_baseline": None,
        "dtype": "bf16" if args.model != "0.5b" else "fp16",
        "data": "synthetic (random-init weights, random token ids / random KV cache)",
        "config": _config(args),
        "cpu_baseline": {"value": rate, "unit": "tok/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": rate, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def _layout_desc(args) -> str:
    from tritonforge_b200.decode import QwenDecoder

    lo, hi = QwenDecoder.COLMAJOR_BATCH
    cm = args.layout == "cm" or (args.layout == "auto" and lo <= args.batch <= hi)
    if not cm:
        return "K-major packed [K/2, N] (the reference's format; mma.sync decode GEMV)"
    return ("tiled column-major, repacked once from the reference's K-major format (tcgen05 decode GEMV) for "
            "projections with K >= 2048; narrower ones K-major")


def _config(args) -> dict:
    tp = args.model != "0.5b"
    par = (f"tp{args.gpus}" if tp else f"replicas{args.gpus}") if args.gpus > 1 else "single"
    if tp and args.gpus > 1:
        par += "+fused-allreduce-rmsnorm" if args.allreduce == "fused" else "+nccl-allreduce"
    return {"workload": f"Qwen2.5-{args.model.upper()}-shaped int4 g128 greedy decode", "model": f"qwen2.5-{args.model}",
            "batch_per_gpu": args.batch, "prompt_len": args.prompt,
            "global_batch": args.batch if tp else args.batch * args.gpus, "parallelism": par,
            "weights": ("int4 group-128, bf16 scales/zeros/activations; embedding, norms and lm_head bf16"
                        if tp else "int4 group-128 (fp16 scales/zeros); embeddings/norms/lm_head fp16"),
            "layout": _layout_desc(args),
            "l2": "per-step working set (int4 weights + lm_head) exceeds the 126 MB L2"}


def gemv_roofline(dec, peak_gbs: float, reps: int = 20, batch_rows: int | None = None) -> dict:
    """Time the step's int4 GEMV launches alone (same shapes, weights and
    inputs) in a CUDA graph; achieved = algorithmic bytes / measured time.
    With `batch_rows`, the same launches on the first rows of the step's
    buffers (the same weights at a smaller batch, 1 for batch-1 decode)."""
    import torch

    from tritonforge_b200 import kernels

    b = dec.buf
    rows = slice(0, batch_rows) if batch_rows else slice(None)
    launches = []  # (x, weights, out, fused gate|up + SwiGLU)
    for L in dec.layers:
        launches += [(b["normed"][rows], L["qkv"], b["qkv"][rows], False),
                     (b["attn"][rows], L["o"], b["o"][rows], False),
                     (b["normed"][rows], L["gu"], b["act"][rows], True),
                     (b["act"][rows], L["down"], b["mlp"][rows], False)]

    def run():
        for x, ql, out, gate_up in launches:
            if gate_up:
                dec._gate_up(x, ql, out)  # the step's own fused launch
            else:
                dec._lin(x, ql, out)

    s = torch.cuda.Stream(dec.dev)
    with torch.cuda.stream(s):
        run()
    torch.cuda.synchronize(dec.dev)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        run()
    g.replay()
    torch.cuda.synchronize(dec.dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(s):
        e0.record(s)
        for _ in range(reps):
            g.replay()
        e1.record(s)
    torch.cuda.synchronize(dec.dev)
    total_us = e0.elapsed_time(e1) * 1e3 / reps
    alg = 0
    kinds = set()
    for x, ql, out, _ in launches:
        m, k = x.shape
        kp, n = ql.scales.shape[0] * ql.group_size, ql.scales.shape[1]
        kinds.add(type(ql).__name__)
        alg += m * k * 2 + kp * n // 2 + 2 * (kp // ql.group_size) * n * 2 + out.numel() * out.element_size()
        if ql.bias is not None:
            alg += n * 2
    achieved = alg / (total_us * 1e-6) / 1e9
    kernel = " + ".join(sorted({"CMLinear": "gemv_int4_cm (tcgen05, tiled column-major weights)",
                                "QuantLinear": "gemv_int4 (mma.sync, K-major weights)"}[k] for k in kinds))
    return {"kernel": kernel, "bound": "hbm", "achieved": achieved,
            "peak": peak_gbs, "unit": "GB/s", "frac": achieved / peak_gbs, "traffic": None,
            "launches_per_step": len(launches), "algorithmic_bytes_per_step": alg,
            "us_per_launch": total_us / len(launches)}


def time_prefill(weights, group, world: int, args, dev) -> dict:
    """Time to first token of one prompt of `args.prefill_len` random token ids
    through QwenDecoder.prefill_tokens (batch 1, K-major projections: every
    projection runs the tcgen05 GEMM at M = prompt length, the library's
    attention covers the prompt, the lm_head + argmax the last position).
    Device-timed with the prompt resident, max over ranks; and end to end with
    the prompt copied from pinned host memory and the first token read back."""
    import torch

    from tritonforge_b200.decode import QwenDecoder

    n = args.prefill_len
    pre = QwenDecoder(weights, batch=1, max_len=n + 8, group=group, fused_allreduce=False, colmajor=False)
    g = torch.Generator().manual_seed(7)
    host = torch.randint(0, weights.embed.shape[0], (1, n), generator=g).pin_memory()
    first = torch.empty(1, dtype=torch.long, pin_memory=True)
    resident = host.to(dev)
    pre.prefill_tokens(resident)  # warm-up: workspaces, kernel attributes, attention backend
    torch.cuda.synchronize(dev)
    reps = max(1, args.prefill_reps)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize(dev)
    e0.record()
    for _ in range(reps):
        pre.prefill_tokens(resident)
    e1.record()
    torch.cuda.synchronize(dev)
    ms = _max_over_ranks(e0.elapsed_time(e1) / reps, world)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize(dev)
    e0.record()
    for _ in range(reps):
        first.copy_(pre.prefill_tokens(host), non_blocking=True)
    e1.record()
    torch.cuda.synchronize(dev)
    e2e_ms = _max_over_ranks(e0.elapsed_time(e1) / reps, world)
    errs = pre.device_errors()
    # projection FLOPs of this rank's shards (2 x rows x K x N per projection)
    flops = sum(2 * n * L[p].packed.shape[0] * 2 * L[p].packed.shape[1]
                for L in pre.layers for p in ("qkv", "o", "gu", "down"))
    pre.release()
    del pre
    torch.cuda.empty_cache()
    if errs:
        raise RuntimeError(f"prefill kernels reported device error bits {errs}")
    peak = _peaks_tensor()
    achieved = flops / (ms / 1000.0) / 1e12
    return {"prompt_tokens": n, "batch": 1, "reps": reps, "ttft_ms": ms, "tok_per_s": n / (ms / 1000.0),
            "e2e_ttft_ms": e2e_ms, "h2d_bytes": host.numel() * 8, "d2h_bytes": 8,
            "projection_tflop_per_gpu": flops / 1e12,
            "projection_tflops_per_gpu": achieved,
            "frac_of_bf16_peak": achieved / peak["bf16_tflops"], "peak_source": peak["source"],
            "note": ("whole prefill time (GEMMs, library attention, RoPE, norms, SwiGLU, lm_head) "
                     "over the projections' FLOPs alone, against the measured cuBLAS bf16 burst peak")}


def run_ours(args) -> None:
    world, rank, local = _dist()
    import torch
    import torch.distributed as dist

    from tritonforge_b200.decode import QwenDecoder

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    tp = args.model != "0.5b"
    cpu_copy = model = None
    parity = prefill = None
    if tp and world > 1 and not args.no_tp_parity:
        # before the timed model is built: the sharded decode of two seeded
        # layers against the same layers decoded on one GPU, on every rank
        from tritonforge_b200.decode import tp_parity

        parity = tp_parity(args.model, dist.group.WORLD, args.batch)
    if tp:
        # tensor parallel over all ranks: synthetic seeded int4 shards generated on each rank
        from tritonforge_b200.decode import QwenWeights

        args.want_cpu = False
        cache_dir = os.path.join(args.weights_cache, f"{args.model}-tp{world}-rank{rank}") if args.weights_cache else None
        if cache_dir and os.path.exists(os.path.join(cache_dir, "manifest.json")):
            weights = QwenWeights.load(cache_dir, device=dev, tp=world, rank=rank)
        else:
            weights = QwenWeights.synthetic(args.model, tp=world, rank=rank, dtype=torch.bfloat16, device=dev,
                                            seed=0)
            if cache_dir:
                weights.save(cache_dir, tp=world, rank=rank)
        group = dist.group.WORLD if world > 1 else None
        if args.prefill_len:
            # before any conversion: the prompt's GEMMs read the K-major layout
            prefill = time_prefill(weights, group, world, args, dev)
        lo, hi = QwenDecoder.COLMAJOR_BATCH
        if args.layout == "cm" or (args.layout == "auto" and lo <= args.batch <= hi):
            weights.to_colmajor()  # in place: one copy of the weights in HBM
        max_len = args.prompt + args.warmup + 2 * args.steps + 8
        dec = QwenDecoder(weights, batch=args.batch, max_len=max_len, group=group,
                          fused_allreduce=args.allreduce == "fused", colmajor=args.layout == "cm")
        dec.fill_cache(args.prompt, seed=1)
    else:
        args.want_cpu = (rank == 0 and world == 1 and not args.no_cpu_baseline)
        model, cpu_copy = build_model(args, dev)
        vocab = model.config.vocab_size
        prompt = prompt_ids(args, vocab, rank)
        max_len = args.prompt + args.warmup + 2 * args.steps + 8
        dec = QwenDecoder(model, batch=args.batch, max_len=max_len,
                          colmajor={"auto": None, "cm": True, "kmajor": False}[args.layout])
        # the whole prompt in one pass: M = batch x prompt rows per projection
        # (the tcgen05 GEMM above 128 rows)
        dec.prefill(prompt)
    dec.capture()
    for _ in range(args.warmup):
        dec.replay()
    torch.cuda.synchronize(dev)
    launches_per_step = dec.launches_per_step()

    # ---- device-timed decode (tokens fed back on the device)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev.index if dev.index is not None else 0) as clocks:
        torch.cuda.nvtx.range_push("timed_decode")  # lets a profiler select exactly the timed steps
        e0.record()
        for _ in range(args.steps):
            dec.graph.replay()
        e1.record()
        torch.cuda.synchronize(dev)
        torch.cuda.nvtx.range_pop()
    if world > 1:
        dist.barrier()
    ms = _max_over_ranks(e0.elapsed_time(e1), world)
    seqs = args.batch if tp else world * args.batch  # TP ranks decode the same sequences
    value = seqs * args.steps / (ms / 1000.0)

    # ---- end to end: per step H2D of the input tokens (pinned) + D2H of the output tokens
    host_in = torch.empty(args.batch, dtype=torch.long, pin_memory=True)
    host_out = torch.empty(args.batch, dtype=torch.long, pin_memory=True)
    host_in.copy_(dec.tokens.cpu())
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    s = torch.cuda.current_stream(dev)
    f0 = torch.cuda.Event(enable_timing=True)
    f1 = torch.cuda.Event(enable_timing=True)
    f0.record(s)
    for _ in range(args.steps):
        dec.tokens.copy_(host_in, non_blocking=True)
        dec.graph.replay()
        host_out.copy_(dec.tokens, non_blocking=True)
        s.synchronize()
        host_in.copy_(host_out)
    f1.record(s)
    torch.cuda.synchronize(dev)
    e2e_ms = _max_over_ranks(f0.elapsed_time(f1), world)
    e2e_value = seqs * args.steps / (e2e_ms / 1000.0)

    # ---- where the step's time goes: each part of the step replayed alone
    # (GEMV launches, attention, reductions + norms, embedding/lm_head/argmax),
    # device-timed, max over ranks; "other" is the step minus their sum (below
    # zero when the parts overlap in the full step: each kernel's prologue runs
    # under the previous one's tail through programmatic dependent launch)
    parts = dec.time_parts()
    breakdown = {k: _max_over_ranks(v, world) for k, v in parts.items()}
    breakdown["step"] = ms / args.steps
    breakdown["other"] = breakdown["step"] - sum(breakdown[k] for k in parts)

    peaks = _peaks()
    roof = gemv_roofline(dec, peaks["hbm_gbs"])
    roof["peak_source"] = peaks["source"]
    roof_m1 = gemv_roofline(dec, peaks["hbm_gbs"], batch_rows=1) if args.batch > 1 else None
    # DRAM traffic: an ncu capture of one GEMV launch (read + write bytes over
    # its algorithmic bytes, committed under profiles/), scaled to the step
    traffic_file = {"gemv_int4 (mma.sync, K-major weights)": "gemv_dram_traffic.json",
                    "gemv_int4_cm (tcgen05, tiled column-major weights)": "gemv_cm_dram_traffic.json"}.get(roof["kernel"])
    try:
        if traffic_file is None:
            raise OSError("projections of both layouts")
        with open(os.path.join(ROOT, "profiles", traffic_file)) as f:
            tr = json.load(f)
        roof["traffic"] = tr["ratio"] * roof["algorithmic_bytes_per_step"]
        roof["traffic_unit"] = "bytes per step"
        roof["traffic_source"] = f"ncu dram bytes / algorithmic bytes = {tr['ratio']:.4f} on {tr['case']}"
    except (OSError, KeyError, ValueError):
        pass

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        if tp:
            dec.release()
            rate, cores, sample, _ = cpu_layer_rate(args, float(args.cpu_budget))
        else:
            from oracle.cpu_decode import cpu_reference_model

            cpu_model = cpu_reference_model(cpu_copy, model)
            rate, cores, _, sample = cpu_decode_rate(cpu_model, prompt, 1000, float(args.cpu_budget))
        cpu = {"value": rate, "unit": "tok/s", "cores": cores, "kind": "port", "sample": sample}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": "strong" if tp else "weak",
            "vs_baseline": None, "dtype": "bf16" if tp else "fp16",
            "data": ("synthetic (random-init int4 weight shards; KV cache of the prompt length filled with random "
                     "values in place of a prefill)") if tp else "synthetic (random-init weights, random token ids)",
            "config": _config(args), "clocks": clocks.summary(),
            "e2e": {"value": e2e_value, "unit": "tok/s", "h2d_bytes_per_step": host_in.numel() * 8,
                    "d2h_bytes_per_step": host_out.numel() * 8},
            "gpu_launches": launches_per_step * args.steps,
            "roofline": roof,
            "cpu_baseline": cpu,
            "step_breakdown_ms": breakdown,
        }
        if roof_m1 is not None:
            # the same step's projections at M = 1 (one decode row, the same weights and layout)
            line["roofline_m1"] = roof_m1
        if parity is not None:
            line["tp_parity"] = parity
        if prefill is not None:
            line["prefill"] = prefill
        print(json.dumps(line), flush=True)
    errs = dec.device_errors()
    if errs:
        raise RuntimeError(f"decode kernels reported device error bits {errs} (a bounded wait gave up)")
    dec.release()
    del dec
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


SWEEP_M = (1, 2, 4, 8, 16, 32, 64, 128, 512, 2048, 8192)
SWEEP_KN = ((3584, 3584), (3584, 512), (3584, 18944), (18944, 3584))  # Qwen2.5-7B q/o, k/v, gate/up, down


def _time_rotating(fns, reps: int = 10) -> float:
    """Median-free mean device time (us) of one call, over `reps` CUDA-graph
    replays of `fns` (one call per rotating input copy)."""
    import torch

    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        for f in fns:
            f()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for f in fns:
            f()
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(s):
        e0.record(s)
        for _ in range(reps):
            g.replay()
        e1.record(s)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) * 1e3 / reps / len(fns)


def kernel_sweep(args) -> None:
    """The reference's kernel benchmark on Qwen2.5-7B shapes (its
    benchmarks/run_kernels.py:27-41 shapes, :48-213 measurements):
    quantized_linear over M x (K, N) x {fp16, bf16}, rmsnorm_residual [M, 3584]
    and swiglu [M, 18944], each point's GB/s (the reference's observable bytes:
    x + packed + scales + zeros + out; 4 M H e + H e; 3 M I e) and TFLOP/s
    against the measured peaks. Weights (and, where affordable, activations)
    rotate over copies whose total exceeds the 126 MB L2, so bytes come from
    HBM; a point whose rotation still fits in L2 says so. At M >= 128 the
    reference's large-M path, dequantise the weight and multiply (cuBLAS), is
    timed beside the native kernel. One JSON object per point to stdout and to
    `--sweep-out`."""
    import torch

    from tritonforge_b200 import _lib, kernels, quant

    peaks = _peaks()
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            tflops_peak = float(json.load(f)["bf16_tflops"])
    except Exception:
        tflops_peak = 1590.0
    dev = torch.device("cuda", 0)
    L2 = 126 * 2 ** 20
    out_f = open(args.sweep_out, "w") if args.sweep_out else None
    ms = [int(v) for v in args.sweep_m.split(",")] if args.sweep_m else SWEEP_M

    def emit(rec):
        rec.update(peak_gbs=peaks["hbm_gbs"], peak_tflops=tflops_peak)
        line = json.dumps(rec)
        print(line, flush=True)
        if out_f:
            out_f.write(line + "\n")
            out_f.flush()

    def sk_grid(m, n, k):
        return int(_lib.load().tf_qlinear_gemm_stream_k_grid(m, n, k))

    g = torch.Generator(device=dev).manual_seed(0)
    for dt in (torch.float16, torch.bfloat16):
        dname = "fp16" if dt == torch.float16 else "bf16"
        for k, n in SWEEP_KN:
            w = torch.randn(n, k, device=dev, generator=g) * 0.02
            p, s, z, _ = quant.quantize_int4_group(w, 128, dt)
            del w
            wbytes = p.numel() + s.numel() * 2 + z.numel() * 2
            copies = max(2, min(64, -(-2 * L2 // wbytes)))
            ws = [(p.clone(), s.clone(), z.clone()) for _ in range(copies)]
            for m in ms:
                x = torch.randn(m, k, device=dev, generator=g).to(dt)
                out = torch.empty(m, n, device=dev, dtype=dt)
                fns = [lambda q=q: kernels.quantized_linear(x, q[0], q[1], q[2], None, 128, out=out) for q in ws]
                us = _time_rotating(fns)
                alg = m * k * 2 + wbytes + m * n * 2
                flops = 2 * m * n * k
                rec = {"op": "quantized_linear", "dtype": dname, "M": m, "K": k, "N": n, "us": us,
                       "gbs": alg / us / 1e3, "tflops": flops / us / 1e6,
                       "regime": ("gemv" if m <= 32 else f"gemv x {-(-m // 32)} row chunks" if m <= 128
                                  else "gemm" if not sk_grid(m, n, k) else f"gemm stream-K x {sk_grid(m, n, k)}"),
                       "l2_resident": copies * wbytes < L2}
                rec["frac_hbm"] = rec["gbs"] / peaks["hbm_gbs"]
                rec["frac_tensor"] = rec["tflops"] / tflops_peak
                if m >= 128:
                    # the reference's large-M path: dequantise every call, then a dense matmul
                    dense = torch.empty(k, n, device=dev, dtype=dt)
                    lib = _lib.load()

                    def ref_path(q):
                        _lib.check(lib.tf_dequantize_int4(q[0].data_ptr(), q[1].data_ptr(), q[2].data_ptr(),
                                                          _lib.dtype_code(dt), dense.data_ptr(), _lib.dtype_code(dt),
                                                          k, n, 128, _lib.stream_ptr(dev)), "dequantize_int4")
                        torch.matmul(x, dense, out=out)
                    rec["dequant_cublas_us"] = _time_rotating([lambda q=q: ref_path(q) for q in ws])
                    rec["speedup_vs_dequant_cublas"] = rec["dequant_cublas_us"] / us
                    del dense
                emit(rec)
                del x, out
            del ws, p, s, z
            torch.cuda.empty_cache()
        for op, width in (("rmsnorm_residual", 3584), ("swiglu", 18944)):
            for m in ms:
                one = m * width * 2
                per_call = (4 * one + width * 2) if op == "rmsnorm_residual" else 3 * one
                copies = max(2, min(64, -(-2 * L2 // per_call)))
                a = [torch.randn(m, width, device=dev, generator=g).to(dt) for _ in range(copies)]
                b = [torch.randn(m, width, device=dev, generator=g).to(dt) for _ in range(copies)]
                o1, o2 = torch.empty(m, width, device=dev, dtype=dt), torch.empty(m, width, device=dev, dtype=dt)
                wn = torch.ones(width, device=dev, dtype=dt)
                if op == "rmsnorm_residual":
                    fns = [lambda i=i: kernels.rmsnorm_residual(a[i], b[i], wn, 1e-6, out=(o1, o2))
                           for i in range(copies)]
                else:
                    fns = [lambda i=i: kernels.swiglu(a[i], b[i], out=o1) for i in range(copies)]
                us = _time_rotating(fns)
                emit({"op": op, "dtype": dname, "M": m, "N": width, "us": us, "gbs": per_call / us / 1e3,
                      "frac_hbm": per_call / us / 1e3 / peaks["hbm_gbs"], "l2_resident": copies * per_call < L2})
                del a, b, o1, o2
            torch.cuda.empty_cache()
    if _lib.workspaces.errors(dev):
        raise SystemExit("a bounded device wait gave up during the sweep")
    if out_f:
        out_f.close()


def profile_case(args) -> None:
    """One kernel on a bounded case, launched three times (the first launches
    are warm-up), for an ncu capture of a single launch:
      gemv / gemv_cm  int4 decode linear [m, k] x [k, n] (K-major mma.sync kernel
                      or tiled column-major tcgen05 kernel), bf16
      gemm            int4 prefill-regime linear, bf16
      attention       decode attention, 72B heads (64 q / 8 kv of 128), batch m,
                      context k positions, bf16
      rmsnorm         rmsnorm_residual over [m, n], bf16
      swiglu          swiglu over [m, n], bf16
      prefill         QwenDecoder.prefill_tokens of an m-token prompt through k
                      Qwen2.5-7B-shaped layers (synthetic int4 weights), bf16
    """
    import torch

    from tritonforge_b200 import _lib, colmajor, kernels, quant

    dt, dev = torch.bfloat16, torch.device("cuda", 0)
    case, m, k, n = args.profile_case, args.m, args.k, args.n
    g = torch.Generator(device=dev).manual_seed(0)
    if case in ("gemv", "gemv_cm", "gemm"):
        w = torch.randn(n, k, device=dev, generator=g) * 0.02
        p, s, z, _ = quant.quantize_int4_group(w, 128, dt)
        del w
        x = torch.randn(m, k, device=dev, generator=g).to(dt)
        out = torch.empty(m, n, device=dev, dtype=dt)
        tiles = colmajor.repack_cm(p) if case == "gemv_cm" else None
        for _ in range(3):
            if tiles is not None:
                colmajor.quantized_linear_cm(x, tiles, s, z, None, 128, out=out)
            else:
                kernels.quantized_linear(x, p, s, z, None, 128, {"regime": case}, out=out)
    elif case == "attention":
        b, hq, hkv, d, ctx = m, 64, 8, 128, k
        t_max = ctx + 64
        kc = torch.randn(b, hkv, t_max, d, device=dev, generator=g, dtype=dt)
        vc = torch.randn(b, hkv, t_max, d, device=dev, generator=g, dtype=dt)
        q = torch.randn(b, hq, d, device=dev, generator=g, dtype=dt)
        out = torch.empty(b, hq * d, device=dev, dtype=dt)
        lens = torch.tensor([ctx, ctx + 1], dtype=torch.int32, device=dev)
        lib = _lib.load()
        for _ in range(3):
            _lib.check(lib.tf_decode_attention(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), out.data_ptr(),
                                               lens.data_ptr() + 4, b, hq, hkv, d, t_max, d ** -0.5,
                                               _lib.dtype_code(dt), _lib.stream_ptr(dev)), "decode_attention")
    elif case == "rmsnorm":
        x = torch.randn(m, n, device=dev, generator=g).to(dt)
        r = torch.randn(m, n, device=dev, generator=g).to(dt)
        w = torch.ones(n, device=dev, dtype=dt)
        normed, summed = torch.empty_like(x), torch.empty_like(x)
        for _ in range(3):
            kernels.rmsnorm_residual(x, r, w, 1e-6, out=(normed, summed))
    elif case == "swiglu":
        a = torch.randn(m, n, device=dev, generator=g).to(dt)
        b_ = torch.randn(m, n, device=dev, generator=g).to(dt)
        out = torch.empty_like(a)
        for _ in range(3):
            kernels.swiglu(a, b_, out=out)
    elif case == "prefill":
        from tritonforge_b200.decode import QwenDecoder, QwenWeights

        w = QwenWeights.synthetic("7b", dtype=dt, device=dev, seed=0, layers=k)
        dec = QwenDecoder(w, 1, m + 8, colmajor=False)
        prompt = torch.randint(0, w.embed.shape[0], (1, m), generator=torch.Generator().manual_seed(0))
        for _ in range(3):
            dec.prefill_tokens(prompt)
        if dec.device_errors():
            raise SystemExit("a bounded device wait gave up")
    else:
        raise SystemExit(f"unknown profile case {case!r}")
    torch.cuda.synchronize(dev)
    if _lib.workspaces.errors(dev):
        raise SystemExit("a bounded device wait gave up")
    print(f"profile case {case} m={m} k={k} n={n} ok", flush=True)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--model", default="72b", choices=["72b", "7b", "0.5b"],
                    help="72b/7b: tensor parallel across the GPUs; 0.5b: transformers model, one replica per GPU")
    ap.add_argument("--batch", type=int, default=None, help="sequences (default 32 for 72b/7b, 8 for 0.5b)")
    ap.add_argument("--prompt", type=int, default=None, help="context length (default 4096 / 2048 / 128)")
    ap.add_argument("--allreduce", choices=["fused", "nccl"], default="fused",
                    help="tensor parallel: fused all-reduce + RMSNorm over peer memory, or NCCL + RMSNorm")
    ap.add_argument("--prefill-len", type=int, default=None,
                    help="prompt tokens of the timed batch-1 prefill (TTFT) of the 7b/72b models; 0 for none "
                         "(default 2048)")
    ap.add_argument("--prefill-reps", type=int, default=2, help="timed prefills (after one warm-up)")
    ap.add_argument("--cpu-budget", type=float, default=20.0, help="seconds of CPU decode for cpu_baseline")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-tp-parity", action="store_true",
                    help="skip the tensor-parallel parity check (two seeded layers, TP-N against one GPU) at N > 1")
    ap.add_argument("--weights-cache", default=None,
                    help="directory of saved int4 shards (one subdirectory per model, TP degree and rank): "
                         "loaded when present, else generated and saved there")
    ap.add_argument("--layout", choices=["auto", "cm", "kmajor"], default="auto",
                    help="int4 weight layout of the decode projections: tiled column-major (tcgen05 kernel), "
                         "the reference's K-major (mma.sync kernel), or auto (column-major for batches 9..128)")
    ap.add_argument("--profile-case", default=None,
                    choices=["gemv", "gemv_cm", "gemm", "attention", "rmsnorm", "swiglu", "prefill"],
                    help="instead of the benchmark: one kernel on a bounded case (--m/--k/--n), for an ncu capture")
    ap.add_argument("--m", type=int, default=32)
    ap.add_argument("--k", type=int, default=8192)
    ap.add_argument("--n", type=int, default=59136)
    ap.add_argument("--sweep", action="store_true",
                    help="instead of the benchmark: the kernel shape sweep on Qwen2.5-7B shapes (one JSON per point)")
    ap.add_argument("--sweep-m", default=None, help="comma-separated M values for --sweep (default: all)")
    ap.add_argument("--sweep-out", default=None, help="also write the sweep's JSON lines to this file")
    args = ap.parse_args()
    if args.profile_case:
        profile_case(args)
        return
    if args.sweep:
        kernel_sweep(args)
        return
    if args.batch is None:
        args.batch = 8 if args.model == "0.5b" else 32
    if args.prompt is None:
        args.prompt = {"72b": 4096, "7b": 2048, "0.5b": 128}[args.model]
    if args.prefill_len is None:
        args.prefill_len = 0 if args.model == "0.5b" else 2048
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
