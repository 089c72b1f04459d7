"""Static-shape Qwen2 decode engine on the B200 kernels.

One decode step for a batch of B sequences is a fixed sequence of launches on
static buffers, so it can be captured once in a CUDA graph and replayed per
token (the reference's end-to-end path is launch-bound: about ten Triton
launches per layer plus transformers' attention, reference
docs/FINAL_REPORT.md:93-99). Per layer:

    rmsnorm_residual(mlp_out_prev, residual)  -> normed, residual      (layer 0: rmsnorm)
    quantized_linear(normed, [q|k|v])          -> qkv                   (one GEMV, bias)
    decode_attention_rope(qkv, cache, pos)     -> attn (q and the new key rotated, K/V appended at pos)
    quantized_linear(attn, o)                  -> o
    rmsnorm_residual(o, residual)              -> normed, residual
    qlinear_swiglu(normed, [gate|up])          -> act = silu(gate) * up (one GEMV, fused epilogue)
    quantized_linear(act, down)                -> mlp_out

then rmsnorm_residual(mlp_out, residual, final_norm), and the lm_head GEMV with
the greedy argmax fused (tf_lm_head_argmax); a step starts with the embedding
gather (tf_embed_gather). The math of each step is the reference patched model's
(reference src/tritonforge/integration/qwen.py:101-152): the end-of-layer
`residual + hidden` of the reference is the `summed` output of the next
rmsnorm_residual (same rounding). q|k|v are the reference's separate
QuantLinear tensors concatenated along N and gate|up interleaved per 64
columns, which changes no value: the fused gate|up kernel rounds each
projection to the model dtype before the SwiGLU, as the reference's separate
launches do. With a tensor-parallel group, o_proj / down_proj leave each
rank's unrounded fp32 partial sum (tf_qlinear_partial); the partials are added
across ranks in fp32 and rounded once, fused with the following
rmsnorm_residual (tf_allreduce_rmsnorm_residual over peer memory, or an NCCL
fp32 all-reduce), so a sharded layer rounds where the single-GPU layer rounds.

The prompt is prefilled through the patched transformers model itself and its
KV cache copied into the static cache.
"""

from __future__ import annotations

import dataclasses

import torch

from . import _lib, kernels
from .colmajor import CMLinear, qlinear_cm_swiglu
from .integration.qwen import QuantLinear


@dataclasses.dataclass
class QwenShape:
    hidden: int
    inter: int
    layers: int
    heads: int
    kv_heads: int
    head_dim: int
    vocab: int
    eps: float = 1e-6
    rope_theta: float = 1000000.0
    tied: bool = True


QWEN25 = {
    "0.5b": QwenShape(896, 4864, 24, 14, 2, 64, 151936, tied=True),
    "7b": QwenShape(3584, 18944, 28, 28, 4, 128, 152064, tied=False),
    "72b": QwenShape(8192, 29568, 80, 64, 8, 128, 152064, tied=False),
}


def hf_config(shape: QwenShape, max_positions: int = 32768):
    from transformers import Qwen2Config

    return Qwen2Config(
        vocab_size=shape.vocab, hidden_size=shape.hidden, intermediate_size=shape.inter,
        num_hidden_layers=shape.layers, num_attention_heads=shape.heads,
        num_key_value_heads=shape.kv_heads, head_dim=shape.head_dim, rms_norm_eps=shape.eps,
        rope_theta=shape.rope_theta, tie_word_embeddings=shape.tied,
        max_position_embeddings=max_positions, use_sliding_window=False)


def random_qwen2(name: str, seed: int = 0, dtype: torch.dtype = torch.float16):
    """Random-init HF Qwen2ForCausalLM of a Qwen2.5 shape (CPU, seeded)."""
    from transformers import Qwen2ForCausalLM

    torch.manual_seed(seed)
    model = Qwen2ForCausalLM(hf_config(QWEN25[name]))
    return model.to(dtype).eval()


def _cat_quant(lins: list[QuantLinear]) -> QuantLinear:
    """Concatenate QuantLinears that share the input along the output dim."""
    packed = torch.cat([l.packed for l in lins], dim=1).contiguous()
    scales = torch.cat([l.scales for l in lins], dim=1).contiguous()
    zeros = torch.cat([l.zeros for l in lins], dim=1).contiguous()
    biases = [l.bias for l in lins]
    bias = None
    if any(b is not None for b in biases):
        bias = torch.cat([b if b is not None else torch.zeros(l.out_features, dtype=scales.dtype,
                                                              device=scales.device)
                          for b, l in zip(biases, lins)]).contiguous()
    return QuantLinear(packed, scales, zeros, lins[0].in_features, sum(l.out_features for l in lins),
                       bias, lins[0].group_size)


def _interleave_quant(gate: QuantLinear, up: QuantLinear) -> QuantLinear:
    """gate and up (no bias) as one QuantLinear whose columns are interleaved
    per 64: [gate 0:64 | up 0:64 | gate 64:128 | ...] (tf_qlinear_swiglu layout)."""
    from .tp import interleave_gate_up

    if gate.bias is not None or up.bias is not None:
        raise ValueError("gate/up projections with a bias are not supported")
    return QuantLinear(interleave_gate_up(gate.packed, up.packed).contiguous(),
                       interleave_gate_up(gate.scales, up.scales).contiguous(),
                       interleave_gate_up(gate.zeros, up.zeros).contiguous(),
                       gate.in_features, 2 * gate.out_features, None, gate.group_size)


@dataclasses.dataclass
class QwenWeights:
    """Everything one rank needs to decode: per-layer int4 projections (q|k|v
    concatenated along N; gate and up interleaved per 64 columns, see
    `_interleave_quant`), norms, embedding, lm_head and rotary tables, with
    this rank's head / intermediate counts."""

    layers: list
    embed: torch.Tensor
    lm_head: torch.Tensor
    final_norm: torch.Tensor
    hidden: int
    inter: int          # this rank's intermediate width
    q_heads: int        # this rank's q heads
    kv_heads: int       # this rank's kv heads
    head_dim: int
    eps: float
    rope_theta: float
    model: object = None  # the patched transformers model (prompt prefill), when there is one

    @property
    def device(self) -> torch.device:
        return self.embed.device

    @property
    def dtype(self) -> torch.dtype:
        return self.embed.dtype

    @classmethod
    def from_hf(cls, model) -> "QwenWeights":
        """From a transformers Qwen2 model patched with quantize=True."""
        cfg = model.config
        inner = model.model
        layers = []
        for layer in inner.layers:
            a, m = layer.self_attn, layer.mlp
            for lin in (a.q_proj, a.k_proj, a.v_proj, a.o_proj, m.gate_proj, m.up_proj, m.down_proj):
                if not isinstance(lin, QuantLinear):
                    raise TypeError("QwenDecoder needs a model patched with quantize=True")
            layers.append({
                "in_norm": layer.input_layernorm.weight.detach(),
                "post_norm": layer.post_attention_layernorm.weight.detach(),
                "qkv": _cat_quant([a.q_proj, a.k_proj, a.v_proj]),
                "o": a.o_proj,
                "gu": _interleave_quant(m.gate_proj, m.up_proj),
                "down": m.down_proj,
            })
        return cls(layers, inner.embed_tokens.weight.detach(), model.lm_head.weight.detach(),
                   inner.norm.weight.detach(), cfg.hidden_size, cfg.intermediate_size,
                   cfg.num_attention_heads, cfg.num_key_value_heads,
                   getattr(cfg, "head_dim", None) or cfg.hidden_size // cfg.num_attention_heads,
                   cfg.rms_norm_eps, getattr(cfg, "rope_theta", 1e6), model)

    @classmethod
    def synthetic(cls, name: str, tp: int = 1, rank: int = 0, dtype: torch.dtype = torch.bfloat16,
                  device=None, seed: int = 0, layers: int | None = None) -> "QwenWeights":
        """Random-init int4 weights of a Qwen2.5 shape, generated directly as
        this rank's tensor-parallel shards (N(0, 0.02) fp32 per shard, int4 g128
        quantised on the GPU; norms 1; embedding and lm_head replicated)."""
        from .tp import TPLayout, synthetic_linear

        shape = QWEN25[name]
        lay = TPLayout(tp, rank, shape.hidden, shape.inter, shape.heads, shape.kv_heads, shape.head_dim)
        device = device or torch.device("cuda", torch.cuda.current_device())
        H, D = shape.hidden, shape.head_dim
        i0, i1 = lay.inter_cols
        il = i1 - i0
        nl = layers or shape.layers
        out = []
        for li in range(nl):
            g = torch.Generator(device=device).manual_seed(seed * 1000003 + li * 131 + rank)
            ones = torch.ones(H, dtype=dtype, device=device)
            out.append({
                "in_norm": ones,
                "post_norm": ones,
                "qkv": synthetic_linear((lay.q_heads + 2 * lay.kv_local) * D, H, g, device, dtype, bias=True),
                "o": synthetic_linear(H, lay.q_heads * D, g, device, dtype),
                "gu": synthetic_linear(2 * il, H, g, device, dtype),
                "down": synthetic_linear(H, il, g, device, dtype),
            })
        g = torch.Generator(device=device).manual_seed(seed * 1000003 + 999_999)
        embed = (torch.randn(shape.vocab, H, generator=g, device=device) * 0.02).to(dtype)
        lm_head = embed if shape.tied else (torch.randn(shape.vocab, H, generator=g, device=device) * 0.02).to(dtype)
        return cls(out, embed, lm_head, torch.ones(H, dtype=dtype, device=device), H, il, lay.q_heads,
                   lay.kv_local, D, shape.eps, shape.rope_theta)


    LINEARS = ("qkv", "o", "gu", "down")

    def colmajor_layers(self, min_k: int = 2048) -> list:
        """The layers with every projection whose input width is at least
        `min_k` in the tiled column-major layout (CMLinear, the tcgen05 decode
        kernel, faster from 9 rows up on wide layers); narrower ones stay
        K-major (the mma.sync kernel wins where a column block has few k
        stages). New layer dicts; the original tensors are not touched."""
        from .colmajor import CMLinear

        out = []
        for L in self.layers:
            d = dict(L)
            for name in self.LINEARS:
                ql = L[name]
                if isinstance(ql, QuantLinear) and ql.packed.shape[0] * 2 >= min_k:
                    d[name] = CMLinear.from_quant(ql)
            out.append(d)
        return out

    def save(self, path: str, tp: int = 1, rank: int = 0) -> None:
        """Write these (K-major) weights, rank `rank` of a `tp`-way shard, to a
        directory: see shard_cache."""
        from .shard_cache import save_weights

        save_weights(self, path, tp, rank)

    @classmethod
    def load(cls, path: str, device=None, tp: int | None = None, rank: int | None = None) -> "QwenWeights":
        """Weights written by `save`, on `device` (default: current CUDA
        device); with `tp`/`rank`, a shard of another degree or rank is refused."""
        from .shard_cache import load_weights

        return load_weights(path, device, tp, rank)

    def to_colmajor(self, min_k: int = 2048) -> "QwenWeights":
        """`colmajor_layers` in place: the K-major packed tensors are dropped
        (memory for one copy of the weights). Shard before converting."""
        for i, d in enumerate(self.colmajor_layers(min_k)):
            self.layers[i] = d
        torch.cuda.empty_cache()
        return self

    def shard(self, tp: int, rank: int) -> "QwenWeights":
        """This rank's tensor-parallel shard of full (tp=1) weights: slices of
        the quantised tensors, bit-identical to quantising the shard alone."""
        from .tp import TPLayout, shard_cols, shard_rows

        if self.q_heads % tp or self.kv_heads % tp:
            raise ValueError(f"tp={tp} must divide q heads {self.q_heads} and kv heads {self.kv_heads}")
        lay = TPLayout(tp, rank, self.hidden, self.inter, self.q_heads, self.kv_heads, self.head_dim)
        D, I = self.head_dim, self.inter
        nq, nkv = self.q_heads * D, self.kv_heads * D
        (q0, q1), (k0, k1), (i0, i1) = lay.q_cols, lay.kv_cols, lay.inter_cols

        def cols(ql: QuantLinear, spans) -> QuantLinear:
            parts = [shard_cols(ql.packed, ql.scales, ql.zeros, ql.bias, a, b) for a, b in spans]
            bias = None if ql.bias is None else torch.cat([p[3] for p in parts]).contiguous()
            return QuantLinear(torch.cat([p[0] for p in parts], 1).contiguous(),
                               torch.cat([p[1] for p in parts], 1).contiguous(),
                               torch.cat([p[2] for p in parts], 1).contiguous(),
                               ql.in_features, sum(b - a for a, b in spans), bias, ql.group_size)

        def rows(ql: QuantLinear, a: int, b: int) -> QuantLinear:
            p, s, z = shard_rows(ql.packed, ql.scales, ql.zeros, a, b, ql.group_size)
            return QuantLinear(p, s, z, b - a, ql.out_features, ql.bias, ql.group_size)

        layers = []
        for L in self.layers:
            layers.append({
                "in_norm": L["in_norm"], "post_norm": L["post_norm"],
                "qkv": cols(L["qkv"], [(q0, q1), (nq + k0, nq + k1), (nq + nkv + k0, nq + nkv + k1)]),
                "o": rows(L["o"], q0, q1),
                "gu": cols(L["gu"], [(2 * i0, 2 * i1)]),  # interleaved: intermediate [i0, i1) is one span
                "down": rows(L["down"], i0, i1),
            })
        return QwenWeights(layers, self.embed, self.lm_head, self.final_norm, self.hidden, i1 - i0,
                           lay.q_heads, lay.kv_local, D, self.eps, self.rope_theta)


def rotary_tables(w: QwenWeights, max_len: int) -> tuple[torch.Tensor, torch.Tensor]:
    """cos/sin [max_len, D] in the model dtype, as transformers' Qwen2 computes them."""
    if w.model is not None:
        inner = w.model.model
        pos = torch.arange(max_len, device=w.device).unsqueeze(0)
        probe = torch.zeros(1, 1, w.hidden, dtype=w.dtype, device=w.device)
        cos, sin = inner.rotary_emb(probe, pos)
        return cos[0].contiguous(), sin[0].contiguous()
    from transformers.models.qwen2.modeling_qwen2 import Qwen2RotaryEmbedding

    cfg = hf_config(QwenShape(w.hidden, w.inter, 1, w.q_heads, w.kv_heads, w.head_dim, 1, w.eps, w.rope_theta))
    rot = Qwen2RotaryEmbedding(cfg).to(w.device)
    pos = torch.arange(max_len, device=w.device).unsqueeze(0)
    cos, sin = rot(torch.zeros(1, 1, 8, dtype=w.dtype, device=w.device), pos)
    return cos[0].contiguous(), sin[0].contiguous()


class QwenDecoder:
    """Batch-B greedy decoder over int4 Qwen2 weights (one rank of a
    tensor-parallel group when `group` is given: the o_proj and down_proj
    outputs are then partial sums, added across ranks by an all-reduce).
    `group` is a torch.distributed process group, or any object with an
    `all_reduce(tensor)` method that sums in place across the ranks."""

    # batches the tcgen05 decode kernel (tiled column-major weights) serves:
    # one launch per 64 rows; at 65..128 rows its two launches still beat four
    # 32-row chunks of the K-major kernel
    COLMAJOR_BATCH = (9, 128)

    def __init__(self, model_or_weights, batch: int, max_len: int, group=None, vocab_parallel: bool | None = None,
                 fused_allreduce: bool | None = None, colmajor: bool | None = None):
        w = model_or_weights if isinstance(model_or_weights, QwenWeights) else QwenWeights.from_hf(model_or_weights)
        self.w = w
        self.model = w.model
        self.group = group
        # Vocab-parallel lm_head (torch.distributed groups only): each rank
        # scores its slice of the vocabulary and the ranks agree on the argmax
        # through an all-gather of (best logit, token id) pairs.
        self.world, self.rank = 1, 0
        if group is not None and not hasattr(group, "all_reduce"):
            import torch.distributed as dist

            self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        self.vocab_parallel = (self.world > 1) if vocab_parallel is None else (vocab_parallel and self.world > 1)
        # Fused all-reduce + residual + RMSNorm over peer memory (tf_allreduce_rmsnorm_residual)
        # in place of an NCCL all-reduce followed by rmsnorm_residual.
        self.fused_allreduce = (self.world > 1) if fused_allreduce is None else (fused_allreduce and self.world > 1)
        self.B, self.T = batch, max_len
        self.H, self.I = w.hidden, w.inter
        self.Hq, self.Hkv, self.D = w.q_heads, w.kv_heads, w.head_dim
        self.eps = w.eps
        # Weight layout: projections already converted (QwenWeights.to_colmajor)
        # are used as they are; otherwise, for batches the tcgen05 decode kernel
        # serves (colmajor=None) or when asked, this decoder converts its own
        # copies of the wide projections.
        lo, hi = self.COLMAJOR_BATCH
        if colmajor is None:
            colmajor = lo <= batch <= hi
        if batch > hi and (colmajor or any(isinstance(L[n], CMLinear) for L in w.layers for n in w.LINEARS)):
            raise ValueError(f"column-major weights serve batches up to {hi} (got {batch})")
        self.layers = w.colmajor_layers() if colmajor else w.layers
        self.final_norm, self.embed, self.lm_head = w.final_norm, w.embed, w.lm_head
        self.vocab = w.lm_head.shape[0]
        self.v0 = 0
        if self.vocab_parallel:
            from .tp import split_even

            self.v0, v1 = split_even(self.vocab, self.world, self.rank)
            self.lm_head = w.lm_head[self.v0:v1].contiguous()
        self.dev, self.dtype = w.device, w.dtype
        self.scale = self.D ** -0.5
        dev, dt, B = self.dev, self.dtype, batch
        self.cos, self.sin = rotary_tables(w, max_len)
        nl = len(self.layers)
        self.k_cache = torch.zeros(nl, B, self.Hkv, max_len, self.D, dtype=dt, device=dev)
        self.v_cache = torch.zeros_like(self.k_cache)
        nqkv = (self.Hq + 2 * self.Hkv) * self.D
        self.tokens = torch.zeros(B, dtype=torch.long, device=dev)
        self.pos = torch.zeros(2, dtype=torch.int32, device=dev)  # [position, length = position + 1]
        self.buf = {
            "x": torch.empty(B, self.H, dtype=dt, device=dev),
            "normed": torch.empty(B, self.H, dtype=dt, device=dev),
            "res_a": torch.empty(B, self.H, dtype=dt, device=dev),
            "res_b": torch.empty(B, self.H, dtype=dt, device=dev),
            "qkv": torch.empty(B, nqkv, dtype=dt, device=dev),
            "q": torch.empty(B, self.Hq, self.D, dtype=dt, device=dev),
            "attn": torch.empty(B, self.Hq * self.D, dtype=dt, device=dev),
            "o": torch.empty(B, self.H, dtype=dt, device=dev),
            "act": torch.empty(B, self.I, dtype=dt, device=dev),
            "mlp": torch.empty(B, self.H, dtype=dt, device=dev),
            "logits": torch.empty(B, self.lm_head.shape[0], dtype=dt, device=dev),
        }
        # Tensor parallel: o_proj / down_proj leave unrounded fp32 partial sums
        # (tf_qlinear_partial), added across ranks in fp32 and rounded once, so
        # a sharded layer rounds exactly where the single-GPU layer does.
        self.tp = group is not None
        if self.fused_allreduce:
            self._setup_symmetric(B)
        elif self.tp:
            self.buf["o_part"] = torch.empty(B, self.H, dtype=torch.float32, device=dev)
            self.buf["mlp_part"] = torch.empty(B, self.H, dtype=torch.float32, device=dev)
        if self.vocab_parallel:
            self.buf["best"] = torch.empty(B, 2, dtype=torch.float32, device=dev)     # (logit, token id)
            self.buf["all_best"] = torch.empty(self.world, B, 2, dtype=torch.float32, device=dev)
        self.graph: torch.cuda.CUDAGraph | None = None
        self._lib = _lib.load()
        self._dt = _lib.dtype_code(dt)

    # ---------------------------------------------------- fused all-reduce
    PAD_SLOT = 64  # first signal-pad slot this decoder uses

    def _setup_symmetric(self, B: int) -> None:
        """Symmetric buffer holding the o_proj and down_proj fp32 partial
        tiles (they alternate, which makes buffer reuse safe without a second
        barrier), peer pointers and signal pads (torch symmetric memory)."""
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm

        n = B * self.H
        sbuf = symm.empty(2 * n, dtype=torch.float32, device=self.dev)
        hdl = symm.rendezvous(sbuf, self.group)
        if hdl.signal_pad_size < 4 * (self.PAD_SLOT + self.world):
            raise RuntimeError("symmetric-memory signal pad too small")
        hdl.get_signal_pad(hdl.rank, (self.PAD_SLOT + self.world,), torch.int32)[self.PAD_SLOT:].zero_()
        self._symm = (sbuf, hdl)
        self.buf["o_part"] = sbuf[:n].view(B, self.H)
        self.buf["mlp_part"] = sbuf[n:].view(B, self.H)
        esz = sbuf.element_size()
        base = int(hdl.offset)  # this tensor's offset inside every rank's buffer
        self._ar_off = {"o": base, "mlp": base + n * esz}
        if any(off % 32 for off in self._ar_off.values()):
            raise RuntimeError(f"symmetric partial tiles not 32-byte aligned: {self._ar_off}")
        self._ar_ctr = torch.zeros(2, dtype=torch.int32, device=self.dev)
        self._ar_err = torch.zeros(1, dtype=torch.int32, device=self.dev)
        torch.cuda.synchronize(self.dev)
        dist.barrier(group=self.group)

    def _ar_norm(self, which: str, res: torch.Tensor, weight: torch.Tensor, normed: torch.Tensor,
                 summed: torch.Tensor) -> None:
        _, hdl = self._symm
        _lib.check(self._lib.tf_allreduce_rmsnorm_residual(
            hdl.buffer_ptrs_dev, hdl.signal_pad_ptrs_dev, self._ar_off[which], self.PAD_SLOT, self.rank, self.world,
            self._ar_ctr.data_ptr(), res.data_ptr(), weight.data_ptr(), _lib.dtype_code(weight.dtype),
            normed.data_ptr(), summed.data_ptr(), self.B, self.H, self.eps, self._dt, _lib.F32,
            self._ar_err.data_ptr(), _lib.stream_ptr(self.dev)), "allreduce_rmsnorm_residual")

    def allreduce_errors(self) -> int:
        """Device error bits of the fused all-reduce (16: a peer's signal did not arrive within 1 s)."""
        return int(self._ar_err.item()) if self.fused_allreduce else 0

    def device_errors(self) -> int:
        """Error bits the decode kernels left on this device: the fused
        all-reduce's word and the int4 kernels' workspace words (a bounded
        wait that gave up after 1 s). 0 means every launch ran to the end;
        anything else means the outputs of some step are not to be trusted."""
        return self.allreduce_errors() | _lib.workspaces.errors(self.dev)

    # ------------------------------------------------------------------ step
    def _lin(self, x: torch.Tensor, ql, out: torch.Tensor) -> torch.Tensor:
        if isinstance(ql, CMLinear):
            return ql(x, out=out)
        return kernels.quantized_linear(x, ql.packed, ql.scales, ql.zeros, ql.bias, ql.group_size, out=out)

    def _lin_partial(self, x: torch.Tensor, ql, out: torch.Tensor) -> None:
        """out (fp32) = x @ W unrounded, no bias: this rank's share of a
        row-parallel projection (tf_qlinear_partial / tf_qlinear_cm_partial)."""
        m, k = x.shape
        cm = isinstance(ql, CMLinear)
        kp = ql.scales.shape[0] * ql.group_size
        n = ql.scales.shape[1]
        need = (self._lib.tf_qlinear_cm_workspace_bytes(m, n, kp) if cm
                else self._lib.tf_qlinear_workspace_bytes(m, n, kp, ql.group_size))
        ws = _lib.workspaces.get(self.dev, need)
        fn = self._lib.tf_qlinear_cm_partial if cm else self._lib.tf_qlinear_partial
        _lib.check(fn(x.data_ptr(), x.stride(0), self._dt, (ql.tiles if cm else ql.packed).data_ptr(),
                      ql.scales.data_ptr(), ql.zeros.data_ptr(), _lib.dtype_code(ql.scales.dtype), out.data_ptr(),
                      out.stride(0), m, n, k, kp, ql.group_size, ws.data_ptr(), ws.numel(),
                      _lib.stream_ptr(self.dev)), "qlinear_partial")

    def _row_parallel(self, x: torch.Tensor, ql, which: str, res: torch.Tensor, weight: torch.Tensor,
                      normed: torch.Tensor, summed: torch.Tensor, parts=None) -> None:
        """o_proj / down_proj followed by the residual add and the next RMSNorm.
        Single GPU: the projection rounds its own output. Tensor parallel: an
        fp32 partial per rank, summed across ranks in fp32 (the fused peer-memory
        kernel, or an NCCL all-reduce), rounded once, then residual + RMSNorm.
        `parts` (a set of step parts, None for all) selects the projection
        ("gemv") and the reduction + norm ("reduce")."""
        b = self.buf
        gemv = parts is None or "gemv" in parts
        reduce = parts is None or "reduce" in parts
        if not self.tp:
            if gemv:
                self._lin(x, ql, b[which])
            if reduce:
                kernels.rmsnorm_residual(b[which], res, weight, self.eps, out=(normed, summed))
            return
        part = b[which + "_part"]
        if gemv:
            self._lin_partial(x, ql, part)
        if not reduce:
            return
        if self.fused_allreduce:
            self._ar_norm(which, res, weight, normed, summed)
            return
        self._all_reduce(part)
        b[which].copy_(part)  # one rounding of the fp32 sum
        kernels.rmsnorm_residual(b[which], res, weight, self.eps, out=(normed, summed))

    def _all_reduce(self, t: torch.Tensor) -> None:
        if self.group is None:
            return
        if hasattr(self.group, "all_reduce"):  # a reducer object (in-process ranks)
            self.group.all_reduce(t)
            return
        import torch.distributed as dist

        dist.all_reduce(t, group=self.group)

    STEP_PARTS = ("gemv", "attention", "reduce", "head")
    HEAD_ROWS = 64  # rows per tf_lm_head_argmax launch

    @torch.no_grad()
    def step(self) -> torch.Tensor:
        """One decode step: consumes self.tokens at self.pos, writes the next
        tokens into self.tokens and advances self.pos (all on device)."""
        return self._step(None)

    def _step(self, parts) -> torch.Tensor:
        """The step's launches, or only those of the given parts (a subset of
        STEP_PARTS: the int4 projections; RoPE + KV append + attention; the
        row-parallel reductions, residual adds and norms; embedding, lm_head and
        argmax), in the step's order on the same buffers, for timing each part
        on its own."""
        def on(p: str) -> bool:
            return parts is None or p in parts

        b = self.buf
        lib, st = self._lib, _lib.stream_ptr(self.dev)
        res, res_next = b["res_a"], b["res_b"]
        if on("head"):
            # x = res = embed[tokens] (the residual stream starts as the embedding)
            _lib.check(lib.tf_embed_gather(self.embed.data_ptr(), self.embed.stride(0), self.tokens.data_ptr(),
                                           b["x"].data_ptr(), b["x"].stride(0), res.data_ptr(), res.stride(0),
                                           self.embed.shape[0], self.embed.shape[1], self.B,
                                           _lib.dtype_code(self.embed.dtype), st), "embed_gather")
        posp = self.pos.data_ptr()
        nl = len(self.layers)
        for li, L in enumerate(self.layers):
            if li == 0 and on("head"):
                kernels.rmsnorm(b["x"], L["in_norm"], self.eps, out=b["normed"])
            if on("gemv"):
                self._lin(b["normed"], L["qkv"], b["qkv"])
            if on("attention"):
                _lib.check(lib.tf_decode_attention_rope(
                    b["qkv"].data_ptr(), b["qkv"].stride(0), self.cos.data_ptr(), self.sin.data_ptr(),
                    self.k_cache[li].data_ptr(), self.v_cache[li].data_ptr(), posp, b["attn"].data_ptr(), self.B,
                    self.Hq, self.Hkv, self.D, self.T, self.scale, self._dt, st), "decode_attention_rope")
            self._row_parallel(b["attn"], L["o"], "o", res, L["post_norm"], b["normed"], res_next, parts)
            res, res_next = res_next, res
            if on("gemv"):
                self._gate_up(b["normed"], L["gu"], b["act"])
            # the next layer's input norm, or the final norm after the last layer
            nxt = self.layers[li + 1]["in_norm"] if li + 1 < nl else self.final_norm
            self._row_parallel(b["act"], L["down"], "mlp", res, nxt, b["normed"], res_next, parts)
            res, res_next = res_next, res
        if on("head"):
            self._head(b["normed"])
        return self.tokens

    def _head(self, x: torch.Tensor) -> None:
        """Logits of the B rows of x, the greedy tokens into self.tokens (or
        this rank's best (logit, id) pairs, then the vocabulary-parallel
        winner) and pos += 1, in one kernel."""
        b = self.buf
        vp = self.vocab_parallel
        rows = self.HEAD_ROWS
        ws = _lib.workspaces.get(self.dev, self._lib.tf_lm_head_workspace_bytes(min(self.B, rows)))
        for r0 in range(0, self.B, rows):
            # up to 64 rows per launch; the last launch advances the position
            n = min(rows, self.B - r0)
            last = r0 + n == self.B
            _lib.check(self._lib.tf_lm_head_argmax(
                x[r0:].data_ptr(), x.stride(0), self.lm_head.data_ptr(), self.lm_head.stride(0),
                self.lm_head.shape[0], self.lm_head.shape[1], n, _lib.dtype_code(self.lm_head.dtype),
                b["logits"][r0:].data_ptr(), b["logits"].stride(0), None if vp else self.tokens[r0:].data_ptr(),
                b["best"][r0:].data_ptr() if vp else None, self.v0 if vp else 0,
                self.pos.data_ptr() if last else None, self.pos.numel() if last else 0,
                ws.data_ptr(), ws.numel(), _lib.stream_ptr(self.dev)), "lm_head_argmax")
        if vp:
            self._vocab_parallel_argmax()

    @torch.no_grad()
    def time_parts(self, reps: int = 10) -> dict:
        """Device time (ms) of each step part replayed alone in a CUDA graph of
        its own (every rank runs the same parts in the same order, so the
        reductions' collectives match); tokens and position are restored."""
        out = {}
        saved = (self.tokens.clone(), self.pos.clone())
        s = torch.cuda.Stream(self.dev)
        s.wait_stream(torch.cuda.current_stream(self.dev))
        for name in self.STEP_PARTS:
            with torch.cuda.stream(s):
                self._step({name})  # outside capture: workspaces and kernel attributes
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                self._step({name})
            g.replay()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            with torch.cuda.stream(s):
                e0.record(s)
                for _ in range(reps):
                    g.replay()
                e1.record(s)
            torch.cuda.synchronize(self.dev)
            out[name] = e0.elapsed_time(e1) / reps
            del g  # a graph holding collectives goes before the process group does
        self.tokens.copy_(saved[0])
        self.pos.copy_(saved[1])
        torch.cuda.synchronize(self.dev)
        return out

    def _vocab_parallel_argmax(self) -> None:
        """Greedy token over the whole vocabulary from each rank's slice of the
        logits. Ties go to the smallest token id, as torch.argmax over the full
        logits does (the first maximum): within a rank the lm_head kernel keeps
        the first, across ranks the lowest rank (whose ids are smaller) wins."""
        import torch.distributed as dist

        b = self.buf
        dist.all_gather_into_tensor(b["all_best"].view(-1, 2), b["best"], group=self.group)
        _lib.check(self._lib.tf_best_of_ranks(b["all_best"].data_ptr(), self.tokens.data_ptr(), self.world, self.B,
                                              _lib.stream_ptr(self.dev)), "best_of_ranks")

    def _gate_up(self, x: torch.Tensor, ql, act: torch.Tensor) -> None:
        """act = silu(x @ Wg) * (x @ Wu) in one int4 linear with the SwiGLU
        fused: tf_qlinear_swiglu on K-major weights (any rows: decode GEMV,
        its 32-row chunks, or the GEMM with a SwiGLU epilogue),
        tf_qlinear_cm_swiglu on column-major weights (64 rows per launch)."""
        m, k = x.shape
        if isinstance(ql, CMLinear):
            qlinear_cm_swiglu(x, ql.tiles, ql.scales, ql.zeros, ql.group_size, out=act)
            return
        if isinstance(ql, QuantLinear):
            n, kp = ql.packed.shape[1], ql.packed.shape[0] * 2
            ws = _lib.workspaces.get(self.dev, self._lib.tf_qlinear_workspace_bytes(m, n, kp, ql.group_size))
            _lib.check(self._lib.tf_qlinear_swiglu(
                x.data_ptr(), x.stride(0), self._dt, ql.packed.data_ptr(), ql.scales.data_ptr(), ql.zeros.data_ptr(),
                _lib.dtype_code(ql.scales.dtype), act.data_ptr(), act.stride(0), m, n, k, kp, ql.group_size,
                ws.data_ptr(), ws.numel(), _lib.stream_ptr(self.dev)), "qlinear_swiglu")
            return
        raise TypeError(f"gate|up projection of unknown type {type(ql).__name__}")

    def launches_per_step(self) -> int:
        """Kernels of this library launched by one step: the embedding gather,
        the first RMSNorm, per layer the four projections (gate|up with its
        SwiGLU fused; column-major projections launch once per 64 rows,
        K-major ones of 33..128 rows once per 32-row chunk), attention and the two residual + norm (or fused
        all-reduce) launches, then the lm_head + argmax and, under
        vocabulary-parallel tensor parallelism, best_of_ranks."""
        n = 2 + -(-self.B // self.HEAD_ROWS) + (1 if self.vocab_parallel else 0)
        for L in self.layers:
            n += 3
            for name in ("qkv", "o", "gu", "down"):
                if isinstance(L[name], CMLinear):
                    n += -(-self.B // 64)
                else:
                    n += -(-self.B // 32) if 32 < self.B <= 128 else 1
        return n

    @torch.no_grad()
    def capture(self) -> None:
        """Capture one decode step in a CUDA graph (after a warm-up step)."""
        s = torch.cuda.Stream(self.dev)
        s.wait_stream(torch.cuda.current_stream(self.dev))
        saved = (self.tokens.clone(), self.pos.clone())
        with torch.cuda.stream(s):
            self.step()  # warm-up: sizes workspaces and sets kernel attributes outside capture
        torch.cuda.current_stream(self.dev).wait_stream(s)
        # the warm-up appended at position `pos`, which the captured step overwrites
        self.tokens.copy_(saved[0])
        self.pos.copy_(saved[1])
        del saved
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            self.step()
        self.graph = g

    def release(self) -> None:
        """Drop the captured graph (before destroying a process group it uses)
        and the symmetric buffer."""
        self.graph = None
        if getattr(self, "_symm", None) is not None:
            torch.cuda.synchronize(self.dev)
            self._symm = None

    def replay(self) -> torch.Tensor:
        if self.graph is None:
            self.capture()
        self.graph.replay()
        return self.tokens

    # ---------------------------------------------------------------- prefill
    @torch.no_grad()
    def prefill(self, prompt: torch.Tensor, chunk: int | None = None) -> torch.Tensor:
        """Run the prompt [B, T0] through the patched transformers model (in
        chunks of `chunk` tokens when given), copy its KV cache into the static
        cache, and set the first generated tokens."""
        if self.model is None:
            raise RuntimeError("prefill needs the transformers model; use fill_cache for synthetic weights")
        if prompt.shape[0] != self.B:
            raise ValueError(f"prompt batch {prompt.shape[0]} != decoder batch {self.B}")
        t0 = prompt.shape[1]
        if t0 >= self.T:
            raise ValueError(f"prompt length {t0} does not fit max_len {self.T}")
        prompt = prompt.to(self.dev)
        if chunk is None:
            out = self.model(prompt, use_cache=True)
            cache = out.past_key_values
        else:
            from transformers import DynamicCache

            cache = DynamicCache()
            for c0 in range(0, t0, chunk):
                out = self.model(prompt[:, c0:c0 + chunk], past_key_values=cache, use_cache=True)
                cache = out.past_key_values
        for li in range(len(self.layers)):
            k, v = _layer_kv(cache, li)
            self.k_cache[li, :, :, :t0].copy_(k)
            self.v_cache[li, :, :, :t0].copy_(v)
        self.tokens.copy_(out.logits[:, -1, :].argmax(-1))
        self.pos.copy_(torch.tensor([t0, t0 + 1], dtype=torch.int32))
        return self.tokens.clone()

    @torch.no_grad()
    def prefill_tokens(self, prompt: torch.Tensor) -> torch.Tensor:
        """Prefill the prompt [B, T0] through this engine's kernels, one
        sequence at a time (M = T0 rows per launch): the embedding gather, the
        norms, every projection through quantized_linear (the tcgen05 GEMM for
        more than 128 rows; under tensor parallelism the row-parallel fp32
        partials are all-reduced and rounded once), RoPE with transformers'
        roundings (q rotated in place, keys and values written to the static
        cache: tf_rope_kv_prefill), causal attention over the prompt (the
        library's scaled-dot-product attention over the cache), the gate|up
        projection with SwiGLU in its epilogue (tf_qlinear_swiglu), and the lm_head +
        argmax of the last positions. Sets the first generated tokens and the
        position; needs the reference's K-major projections (QuantLinear; the
        column-major kernel is a decode kernel, 64 rows per launch)."""
        import torch.nn.functional as F

        if prompt.shape[0] != self.B:
            raise ValueError(f"prompt batch {prompt.shape[0]} != decoder batch {self.B}")
        t0 = prompt.shape[1]
        if t0 < 1 or t0 >= self.T:
            raise ValueError(f"prompt length {t0} does not fit max_len {self.T}")
        for L in self.layers:
            if not all(isinstance(L[n], QuantLinear) for n in ("qkv", "o", "gu", "down")):
                raise RuntimeError("prefill_tokens needs K-major projections (QwenDecoder(..., colmajor=False))")
        prompt = prompt.to(self.dev, torch.long)
        dt, dev, H, D = self.embed.dtype, self.dev, self.H, self.D
        hq, hkv = self.Hq * D, self.Hkv * D
        lib, st = self._lib, _lib.stream_ptr(self.dev)

        def buf(*shape, dtype=dt):
            return torch.empty(*shape, dtype=dtype, device=dev)

        x, res_a, res_b, normed = buf(t0, H), buf(t0, H), buf(t0, H), buf(t0, H)
        qkv, o, act = buf(t0, hq + 2 * hkv), buf(t0, H), buf(t0, self.I)
        part = buf(t0, H, dtype=torch.float32) if self.tp else None
        last = buf(self.B, H)
        code = _lib.dtype_code(dt)

        def row_parallel(xin, ql, weight, res, res_next):
            if self.tp:
                self._lin_partial(xin, ql, part)
                self._all_reduce(part)
                o.copy_(part)  # one rounding of the fp32 sum
            else:
                self._lin(xin, ql, o)
            kernels.rmsnorm_residual(o, res, weight, self.eps, out=(normed, res_next))

        nl = len(self.layers)
        for b in range(self.B):
            toks = prompt[b].contiguous()
            res, res_next = res_a, res_b
            _lib.check(lib.tf_embed_gather(self.embed.data_ptr(), self.embed.stride(0), toks.data_ptr(), x.data_ptr(),
                                           H, res.data_ptr(), H, self.embed.shape[0], H, t0,
                                           _lib.dtype_code(self.embed.dtype), st), "embed_gather")
            kernels.rmsnorm(x, self.layers[0]["in_norm"], self.eps, out=normed)
            for li, L in enumerate(self.layers):
                self._lin(normed, L["qkv"], qkv)
                kc, vc = self.k_cache[li, b], self.v_cache[li, b]
                _lib.check(lib.tf_rope_kv_prefill(qkv.data_ptr(), qkv.stride(0), qkv.data_ptr(), qkv.stride(0),
                                                  self.cos.data_ptr(), self.sin.data_ptr(), kc.data_ptr(),
                                                  vc.data_ptr(), t0, self.Hq, self.Hkv, D, self.T, code, st),
                           "rope_kv_prefill")
                q = qkv[:, :hq].view(t0, self.Hq, D).transpose(0, 1)[None]
                a = F.scaled_dot_product_attention(q, kc[None, :, :t0], vc[None, :, :t0], is_causal=True,
                                                   scale=self.scale, enable_gqa=True)
                attn = a[0].transpose(0, 1).reshape(t0, hq)
                row_parallel(attn, L["o"], L["post_norm"], res, res_next)
                res, res_next = res_next, res
                self._gate_up(normed, L["gu"], act)  # gate|up GEMM with SwiGLU in its epilogue
                nxt = self.layers[li + 1]["in_norm"] if li + 1 < nl else self.final_norm
                row_parallel(act, L["down"], nxt, res, res_next)
                res, res_next = res_next, res
            last[b].copy_(normed[t0 - 1])
        self.pos.copy_(torch.tensor([t0 - 1, t0], dtype=torch.int32))  # the head advances it to [t0, t0 + 1]
        self._head(last)
        return self.tokens.clone()

    @torch.no_grad()
    def fill_cache(self, length: int, seed: int = 0) -> None:
        """Stand-in for a prompt prefill on synthetic weights: random K/V
        (N(0, 1)) for the first `length` positions and random current tokens.
        The decode steps that follow attend over all `length` positions."""
        if length >= self.T:
            raise ValueError(f"length {length} does not fit max_len {self.T}")
        g = torch.Generator(device=self.dev).manual_seed(seed)
        for li in range(len(self.layers)):
            self.k_cache[li, :, :, :length].normal_(generator=g)
            self.v_cache[li, :, :, :length].normal_(generator=g)
        self.tokens.copy_(torch.randint(0, self.embed.shape[0], (self.B,), generator=g, device=self.dev))
        self.pos.copy_(torch.tensor([length, length + 1], dtype=torch.int32))

    @torch.no_grad()
    def generate(self, prompt: torch.Tensor, new_tokens: int, use_graph: bool = True) -> torch.Tensor:
        """Greedy decode: returns [B, new_tokens] token ids (the first from prefill)."""
        toks = [self.prefill(prompt)]
        for _ in range(new_tokens - 1):
            toks.append((self.replay() if use_graph else self.step()).clone())
        return torch.stack(toks, dim=1)


def _layer_kv(cache, li: int):
    """(key, value) [B, Hkv, T, D] of layer li from a transformers cache."""
    if hasattr(cache, "layers"):
        layer = cache.layers[li]
        return layer.keys, layer.values
    if hasattr(cache, "key_cache"):
        return cache.key_cache[li], cache.value_cache[li]
    return cache[li][0], cache[li][1]


# Bounds on the logits of two decodes of the same bf16 weights whose only
# difference is the fp32 summation order (max beyond one ulp of each logit, and
# mean, over the logit RMS): the measured noise floor of that effect without any
# tensor parallelism (two single-GPU decodes through different GEMV kernels)
# reaches 4.7% max and 0.58% mean; these are that floor with headroom.
DECODE_MAX_TOL = 6e-2
DECODE_MEAN_TOL = 1e-2


@torch.no_grad()
def _row_parallel_op_error(name: str, ref: "QwenDecoder", dec: "QwenDecoder", world: int, rank: int,
                           seed: int) -> float:
    """The sharded row-parallel op against the single-GPU op on identical
    inputs: for o_proj and down_proj of layer 0, seeded x [B, K] and residual
    [B, H], every rank runs its K-shard through the tensor-parallel path (fp32
    partial, the group's reduction, residual + RMSNorm) and `ref` runs the
    whole projection then rmsnorm_residual. Returns the largest error of
    `summed` and `normed` beyond their own roundings after the sum (one and
    two bf16 ulps), over their RMS (the per-kernel contract is 2e-2 for bf16)."""
    from .tp import TPLayout

    shape = QWEN25[name]
    lay = TPLayout(world, rank, shape.hidden, shape.inter, shape.heads, shape.kv_heads, shape.head_dim)
    B, H, dev = dec.B, dec.H, dec.dev
    worst = 0.0
    for key, which, (k0, k1), k_full in (("o", "o", lay.q_cols, shape.heads * shape.head_dim),
                                          ("down", "mlp", lay.inter_cols, shape.inter)):
        g = torch.Generator(device=dev).manual_seed(seed * 31 + len(key))
        x = torch.randn(B, k_full, generator=g, device=dev).to(dec.dtype)
        res = torch.randn(B, H, generator=g, device=dev).to(dec.dtype)
        w = torch.ones(H, dtype=dec.dtype, device=dev)
        want_o = torch.empty(B, H, dtype=dec.dtype, device=dev)
        ref._lin(x, ref.layers[0][key], want_o)
        want_n, want_s = kernels.rmsnorm_residual(want_o, res, w, dec.eps)
        normed, summed = torch.empty_like(res), torch.empty_like(res)
        dec._row_parallel(x[:, k0:k1].contiguous(), dec.layers[0][key], which, res, w, normed, summed)
        # beyond the outputs' own roundings after the sum (summed: one; normed: two), whose
        # one-ulp flips the fp32 summation order of the shards can move
        for got, want, ulps in ((summed, want_s, 1), (normed, want_n, 2)):
            wf = want.float()
            ulp = torch.ldexp(torch.ones_like(wf), torch.frexp(wf)[1] - 8)
            rms = float(wf.pow(2).mean().sqrt())
            worst = max(worst, float(((got.float() - wf).abs() - ulps * ulp).clamp_min(0).max()) / rms)
    torch.cuda.synchronize(dev)
    return worst


@torch.no_grad()
def tp_parity(name: str, group, batch: int, layers: int = 2, steps: int = 4, seed: int = 7,
              context: int = 40) -> dict:
    """Tensor-parallel decode against a single-GPU decode of the same weights.

    Every rank builds the same full `layers`-layer weights of the Qwen2.5
    shape `name` (seeded), decodes them alone (tp=1) and decodes its own shard
    with the group (the engine's tensor-parallel path, fused all-reduce), both
    from the same random KV cache of `context` positions, for `steps` greedy
    steps fed the same tokens. Returns max(|logits_tp - logits_tp1| - one bf16
    ulp of the tp=1 logit) / RMS over all steps and ranks' vocabulary slices
    (a logit is itself rounded to bf16, and near 5 x RMS one ulp is ~2.6% of
    the RMS; the raw maximum is reported too), whether the greedy tokens agree,
    the largest reference top-2 gap among rows whose tokens differ (a genuine
    near-tie when within 2e-2 x RMS), whether all ranks produced the same
    tokens, and the device error bits of both decoders."""
    import torch.distributed as dist

    world, rank = dist.get_world_size(group), dist.get_rank(group)
    dev = torch.device("cuda", torch.cuda.current_device())
    full = QwenWeights.synthetic(name, tp=1, rank=0, dtype=torch.bfloat16, device=dev, seed=seed, layers=layers)
    t_max = context + steps + 8
    ref = QwenDecoder(full, batch, t_max)
    ref.fill_cache(context, seed=seed + 1)
    dec = QwenDecoder(full.shard(world, rank), batch, t_max, group=group)
    h = dec.Hkv
    dec.k_cache.copy_(ref.k_cache[:, :, rank * h:(rank + 1) * h])
    dec.v_cache.copy_(ref.v_cache[:, :, rank * h:(rank + 1) * h])
    dec.tokens.copy_(ref.tokens)
    dec.pos.copy_(ref.pos)
    op_err = _row_parallel_op_error(name, ref, dec, world, rank, seed)
    dec.capture()
    v0, nv = dec.v0, dec.lm_head.shape[0]
    worst, raw, mean, same, tie_gap, ranks_same = 0.0, 0.0, 0.0, True, 0.0, True
    for _ in range(steps):
        ref.step()
        dec.graph.replay()
        want = ref.buf["logits"][:, v0:v0 + nv].float()
        rms = float(ref.buf["logits"].float().pow(2).mean().sqrt())
        diff = (dec.buf["logits"].float() - want).abs()
        # a logit is a bf16 value: one ulp of it is its own rounding, allowed on top of the tolerance
        ulp = torch.ldexp(torch.ones_like(want), torch.frexp(want)[1] - 8)
        worst = max(worst, float((diff - ulp).clamp_min(0).max()) / rms)
        raw = max(raw, float(diff.max()) / rms)
        mean = max(mean, float(diff.mean()) / rms)
        diff = (dec.tokens != ref.tokens).nonzero().flatten()
        if diff.numel():
            same = False
            r32 = ref.buf["logits"].float()
            gap = float((r32[diff, ref.tokens[diff]] - r32[diff, dec.tokens[diff]]).max()) / rms
            tie_gap = max(tie_gap, gap)
        gathered = [torch.empty_like(dec.tokens) for _ in range(world)]
        dist.all_gather(gathered, dec.tokens, group=group)
        ranks_same &= all(torch.equal(gathered[0], t) for t in gathered)
        dec.tokens.copy_(ref.tokens)  # both decodes continue from the same tokens
    errs = dec.device_errors() | ref.device_errors()
    stats = torch.tensor([worst, 0.0 if same else 1.0, tie_gap, 0.0 if ranks_same else 1.0, float(errs), raw,
                          mean, op_err], dtype=torch.float64, device=dev)
    dist.all_reduce(stats, op=dist.ReduceOp.MAX, group=group)
    dec.release()
    del dec, ref, full
    torch.cuda.empty_cache()
    op, worst, mean, tie = float(stats[7]), float(stats[0]), float(stats[6]), float(stats[2])
    return {"model": name, "layers": layers, "steps": steps, "batch": batch, "context": context,
            # the sharded op (o_proj / down_proj partials, fused all-reduce, residual + RMSNorm) on
            # identical inputs against the single-GPU op: the per-kernel contract
            "op_max_err_over_rms": op, "op_tolerance": 2e-2,
            # whole decodes: logits after `layers` layers, beyond one bf16 ulp of each logit, and the
            # mean; bounded by the summation-order noise floor of a bf16 decode
            "logits_max_err_over_rms": worst, "logits_max_abs_err_over_rms": float(stats[5]),
            "logits_mean_err_over_rms": mean, "logits_tolerance": {"max": DECODE_MAX_TOL, "mean": DECODE_MEAN_TOL},
            "tokens_equal": stats[1].item() == 0.0, "near_tie_gap_over_rms": tie,
            "ranks_identical": stats[3].item() == 0.0, "device_errors": int(stats[4]),
            "ok": op <= 2e-2 and worst <= DECODE_MAX_TOL and mean <= DECODE_MEAN_TOL and tie <= 2e-2
            and stats[3].item() == 0.0
            and int(stats[4]) == 0}
