"""Static-shape Qwen2 decode engine on the B200 kernels.

One decode step for a batch of B sequences is a fixed sequence of launches on
static buffers, so it can be captured once in a CUDA graph and replayed per
token (the reference's end-to-end path is launch-bound: about ten Triton
launches per layer plus transformers' attention, reference
docs/FINAL_REPORT.md:93-99). Per layer:

    rmsnorm_residual(mlp_out_prev, residual)  -> normed, residual      (layer 0: rmsnorm)
    quantized_linear(normed, [q|k|v])          -> qkv                   (one GEMV, bias)
    rope_kv_append(qkv)                        -> q rotated, K/V cache at pos
    decode_attention(q, cache, len=pos+1)      -> attn
    quantized_linear(attn, o)                  -> o
    rmsnorm_residual(o, residual)              -> normed, residual
    quantized_linear(normed, [gate|up])        -> gu                    (one GEMV)
    swiglu(gu[:, :I], gu[:, I:])               -> act
    quantized_linear(act, down)                -> mlp_out

then rmsnorm_residual(mlp_out, residual, final_norm), the tied fp16 lm_head
(cuBLAS) and argmax. The math of each step is the reference patched model's
(reference src/tritonforge/integration/qwen.py:101-152): the end-of-layer
`residual + hidden` of the reference is the `summed` output of the next
rmsnorm_residual (same rounding). q|k|v and gate|up are the reference's
separate QuantLinear tensors concatenated along N, which changes no value.

The prompt is prefilled through the patched transformers model itself and its
KV cache copied into the static cache.
"""

from __future__ import annotations

import dataclasses

import torch

from . import _lib, kernels
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


class QwenDecoder:
    """Batch-B greedy decoder over a patched (int4 QuantLinear) Qwen2 model."""

    def __init__(self, model, batch: int, max_len: int):
        cfg = model.config
        self.model = model
        self.B = batch
        self.T = max_len
        self.H = cfg.hidden_size
        self.I = cfg.intermediate_size
        self.Hq = cfg.num_attention_heads
        self.Hkv = cfg.num_key_value_heads
        self.D = getattr(cfg, "head_dim", None) or self.H // self.Hq
        self.eps = cfg.rms_norm_eps
        inner = model.model
        self.dev = inner.embed_tokens.weight.device
        self.dtype = inner.embed_tokens.weight.dtype
        self.layers = []
        for layer in inner.layers:
            a, m = layer.self_attn, layer.mlp
            for lin in (a.q_proj, a.k_proj, a.v_proj, a.o_proj, m.gate_proj, m.up_proj, m.down_proj):
                if not isinstance(lin, QuantLinear):
                    raise TypeError("QwenDecoder needs a model patched with quantize=True")
            self.layers.append({
                "in_norm": layer.input_layernorm.weight.detach(),
                "post_norm": layer.post_attention_layernorm.weight.detach(),
                "qkv": _cat_quant([a.q_proj, a.k_proj, a.v_proj]),
                "o": a.o_proj,
                "gu": _cat_quant([m.gate_proj, m.up_proj]),
                "down": m.down_proj,
            })
        self.final_norm = inner.norm.weight.detach()
        self.embed = inner.embed_tokens.weight.detach()
        self.lm_head = model.lm_head.weight.detach()
        self.scale = self.D ** -0.5
        dev, dt, B = self.dev, self.dtype, batch
        # rotary tables [T, D] exactly as transformers computes them
        pos = torch.arange(max_len, device=dev).unsqueeze(0)
        probe = torch.zeros(1, 1, self.H, dtype=dt, device=dev)
        cos, sin = inner.rotary_emb(probe, pos)
        self.cos = cos[0].contiguous()
        self.sin = sin[0].contiguous()
        nl = len(self.layers)
        self.k_cache = torch.zeros(nl, B, self.Hkv, max_len, self.D, dtype=dt, device=dev)
        self.v_cache = torch.zeros_like(self.k_cache)
        # static step buffers
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
            "gu": torch.empty(B, 2 * self.I, dtype=dt, device=dev),
            "act": torch.empty(B, self.I, dtype=dt, device=dev),
            "mlp": torch.empty(B, self.H, dtype=dt, device=dev),
            "logits": torch.empty(B, self.lm_head.shape[0], dtype=dt, device=dev),
        }
        self.graph: torch.cuda.CUDAGraph | None = None
        self._lib = _lib.load()
        self._dt = _lib.dtype_code(dt)

    # ------------------------------------------------------------------ step
    def _lin(self, x: torch.Tensor, ql: QuantLinear, out: torch.Tensor) -> torch.Tensor:
        return kernels.quantized_linear(x, ql.packed, ql.scales, ql.zeros, ql.bias, ql.group_size, out=out)

    @torch.no_grad()
    def step(self) -> torch.Tensor:
        """One decode step: consumes self.tokens at self.pos, writes the next
        tokens into self.tokens and advances self.pos (all on device)."""
        b = self.buf
        lib, st = self._lib, _lib.stream_ptr(self.dev)
        torch.index_select(self.embed, 0, self.tokens, out=b["x"])
        res, res_next = b["res_a"], b["res_b"]
        posp = self.pos.data_ptr()
        lenp = posp + 4
        for li, L in enumerate(self.layers):
            if li == 0:
                kernels.rmsnorm(b["x"], L["in_norm"], self.eps, out=b["normed"])
                res.copy_(b["x"])
            else:
                kernels.rmsnorm_residual(b["mlp"], res, L["in_norm"], self.eps, out=(b["normed"], res_next))
                res, res_next = res_next, res
            self._lin(b["normed"], L["qkv"], b["qkv"])
            _lib.check(lib.tf_rope_kv_append(
                b["qkv"].data_ptr(), b["qkv"].stride(0), b["q"].data_ptr(), self.cos.data_ptr(),
                self.sin.data_ptr(), self.k_cache[li].data_ptr(), self.v_cache[li].data_ptr(), posp,
                self.B, self.Hq, self.Hkv, self.D, self.T, self._dt, st), "rope_kv_append")
            _lib.check(lib.tf_decode_attention(
                b["q"].data_ptr(), self.k_cache[li].data_ptr(), self.v_cache[li].data_ptr(),
                b["attn"].data_ptr(), lenp, self.B, self.Hq, self.Hkv, self.D, self.T, self.scale,
                self._dt, st), "decode_attention")
            self._lin(b["attn"], L["o"], b["o"])
            kernels.rmsnorm_residual(b["o"], res, L["post_norm"], self.eps, out=(b["normed"], res_next))
            res, res_next = res_next, res
            self._lin(b["normed"], L["gu"], b["gu"])
            gu = b["gu"]
            _lib.check(lib.tf_swiglu_strided(
                gu.data_ptr(), gu.data_ptr() + self.I * gu.element_size(), b["act"].data_ptr(), self.B, self.I,
                gu.stride(0), gu.stride(0), b["act"].stride(0), self._dt, st), "swiglu")
            self._lin(b["act"], L["down"], b["mlp"])
        kernels.rmsnorm_residual(b["mlp"], res, self.final_norm, self.eps, out=(b["normed"], res_next))
        torch.matmul(b["normed"], self.lm_head.t(), out=b["logits"])
        torch.argmax(b["logits"], dim=-1, out=self.tokens)
        self.pos.add_(1)
        return self.tokens

    @torch.no_grad()
    def capture(self) -> None:
        """Capture one decode step in a CUDA graph (after a warm-up step)."""
        s = torch.cuda.Stream(self.dev)
        s.wait_stream(torch.cuda.current_stream(self.dev))
        saved = (self.tokens.clone(), self.pos.clone(), self.k_cache.clone(), self.v_cache.clone())
        with torch.cuda.stream(s):
            self.step()  # warm-up: sizes workspaces and sets kernel attributes outside capture
        torch.cuda.current_stream(self.dev).wait_stream(s)
        self.tokens.copy_(saved[0])
        self.pos.copy_(saved[1])
        self.k_cache.copy_(saved[2])
        self.v_cache.copy_(saved[3])
        del saved
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            self.step()
        self.graph = g

    def replay(self) -> torch.Tensor:
        if self.graph is None:
            self.capture()
        self.graph.replay()
        return self.tokens

    # ---------------------------------------------------------------- prefill
    @torch.no_grad()
    def prefill(self, prompt: torch.Tensor) -> torch.Tensor:
        """Run the prompt [B, T0] through the patched model, copy its KV cache
        into the static cache, and set the first generated tokens."""
        if prompt.shape[0] != self.B:
            raise ValueError(f"prompt batch {prompt.shape[0]} != decoder batch {self.B}")
        t0 = prompt.shape[1]
        if t0 >= self.T:
            raise ValueError(f"prompt length {t0} does not fit max_len {self.T}")
        out = self.model(prompt.to(self.dev), use_cache=True)
        cache = out.past_key_values
        for li in range(len(self.layers)):
            k, v = _layer_kv(cache, li)
            self.k_cache[li, :, :, :t0].copy_(k)
            self.v_cache[li, :, :, :t0].copy_(v)
        self.tokens.copy_(out.logits[:, -1, :].argmax(-1))
        self.pos.copy_(torch.tensor([t0, t0 + 1], dtype=torch.int32))
        return self.tokens.clone()

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
