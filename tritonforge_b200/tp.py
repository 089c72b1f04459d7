"""Tensor-parallel sharding of the Qwen2 int4 decode path (no reference
counterpart: the reference is single-GPU).

Megatron-style split, one rank per GPU:

* column-parallel (shard the output dim N): q_proj by q heads, k_proj/v_proj
  by kv heads, gate_proj/up_proj by 128-wide intermediate groups;
* row-parallel (shard the input dim K on 128-group boundaries): o_proj over
  the rank's q heads, down_proj over the rank's intermediate groups; their
  outputs are partial sums that an all-reduce (NCCL over NVLink) adds.

Shards are slices of the quantised tensors: K-major `packed[K/2, N]` and
`scales/zeros[K/128, N]` slice by columns (column-parallel) or by rows of
whole groups (row-parallel), so quantising before or after sharding gives the
same bits. Intermediate sizes that are not a multiple of tp*128 split unevenly
(Qwen2.5-72B: 29568 = 231 groups -> TP8 ranks get 29,29,29,29,29,29,29,28).
"""

from __future__ import annotations

import dataclasses

import torch

GROUP = 128


def split_even(total: int, parts: int, rank: int) -> tuple[int, int]:
    """[start, end) of `rank`'s share when `total` units are split as evenly
    as possible, the first `total % parts` ranks taking one extra."""
    if parts <= 0 or not 0 <= rank < parts:
        raise ValueError(f"bad rank {rank} of {parts}")
    base, extra = divmod(total, parts)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


@dataclasses.dataclass(frozen=True)
class TPLayout:
    """Per-rank sizes of a Qwen2 shape under tensor parallelism `tp`."""

    tp: int
    rank: int
    hidden: int
    inter: int
    heads: int
    kv_heads: int
    head_dim: int

    def __post_init__(self):
        if self.heads % self.tp or self.kv_heads % self.tp:
            raise ValueError(f"tp={self.tp} must divide q heads {self.heads} and kv heads {self.kv_heads}")
        if self.inter % GROUP:
            raise ValueError("intermediate size must be a multiple of 128")

    @property
    def q_heads(self) -> int:
        return self.heads // self.tp

    @property
    def kv_local(self) -> int:
        return self.kv_heads // self.tp

    @property
    def q_cols(self) -> tuple[int, int]:
        w = self.q_heads * self.head_dim
        return self.rank * w, (self.rank + 1) * w

    @property
    def kv_cols(self) -> tuple[int, int]:
        w = self.kv_local * self.head_dim
        return self.rank * w, (self.rank + 1) * w

    @property
    def inter_cols(self) -> tuple[int, int]:
        g0, g1 = split_even(self.inter // GROUP, self.tp, self.rank)
        return g0 * GROUP, g1 * GROUP


def shard_cols(packed: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor, bias, c0: int, c1: int):
    """Column-parallel shard of a quantised linear (output columns [c0, c1))."""
    b = None if bias is None else bias[c0:c1].contiguous()
    return (packed[:, c0:c1].contiguous(), scales[:, c0:c1].contiguous(), zeros[:, c0:c1].contiguous(), b)


def shard_rows(packed: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor, k0: int, k1: int,
               group: int = GROUP):
    """Row-parallel shard (input rows [k0, k1), whole groups) of a quantised linear."""
    if k0 % group or k1 % group:
        raise ValueError("row shards must start and end on group boundaries")
    return (packed[k0 // 2:k1 // 2].contiguous(), scales[k0 // group:k1 // group].contiguous(),
            zeros[k0 // group:k1 // group].contiguous())


def synthetic_linear(n: int, k: int, gen: torch.Generator, device, dtype, std: float = 0.02, bias: bool = False):
    """Random fp32 weight [n, k] ~ N(0, std) quantised with the int4 g128 quantizer."""
    from .integration.qwen import QuantLinear
    from .quant import quantize_int4_group

    w = torch.randn(n, k, generator=gen, device=device, dtype=torch.float32).mul_(std)
    packed, scales, zeros, _ = quantize_int4_group(w, GROUP, dtype)
    del w
    b = (torch.randn(n, generator=gen, device=device) * std).to(dtype) if bias else None
    return QuantLinear(packed, scales, zeros, k, n, b, GROUP)


def local_best(logits: torch.Tensor, v0: int, out: torch.Tensor, arg: torch.Tensor) -> torch.Tensor:
    """(best logit, global token id) per row of this rank's vocabulary slice
    `logits` [B, V_local] (ids offset by v0), as fp32 pairs in `out` [B, 2];
    the first maximum within the slice wins, as in torch.argmax."""
    torch.argmax(logits, dim=-1, out=arg)
    out[:, :1].copy_(torch.gather(logits, 1, arg.unsqueeze(1)))  # exact: fp16/bf16 values fit in fp32
    out[:, 1].copy_(arg).add_(v0)                               # exact: ids < 2^24
    return out


def best_of_ranks(all_best: torch.Tensor) -> torch.Tensor:
    """Token ids [B] (fp32) from every rank's (best logit, id) pairs
    [world, B, 2], ranks holding consecutive vocabulary slices in rank order:
    the largest logit wins and ties go to the lowest rank, whose ids are the
    smallest, so the result equals torch.argmax over the whole vocabulary."""
    win = torch.argmax(all_best[:, :, 0], dim=0)
    return torch.gather(all_best[:, :, 1], 0, win.unsqueeze(0)).squeeze(0)


def interleave_gate_up(gate: torch.Tensor, up: torch.Tensor, block: int = 64) -> torch.Tensor:
    """Columns of gate [R, I] and up [R, I] interleaved per `block` columns:
    [gate 0:64 | up 0:64 | gate 64:128 | up 64:128 | ...] (the layout the fused
    gate|up + SwiGLU decode kernel reads, one 128-column block per CTA)."""
    r, i = gate.shape
    if up.shape != gate.shape or i % block:
        raise ValueError("gate and up must have the same shape with a multiple of the block of columns")
    return torch.stack([gate.reshape(r, i // block, block), up.reshape(r, i // block, block)], dim=2).reshape(r, 2 * i)
