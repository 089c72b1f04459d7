"""CPU restatement of the reference's int4 Qwen2 decode path (TEST ORACLE ONLY;
used by the tests and by bench.py's cpu_baseline / --impl reference legs).

The reference's CPU-capable end-to-end path is transformers' Qwen2 model with
its int4 QuantLinear on the dequantize-then-matmul branch
(reference src/tritonforge/integration/qwen.py:91-97: dequantize the whole
weight to the activation dtype every call, `x @ W[:K]`, `+ bias`), norms as
transformers' RMSNorm and the MLP activation as `reference.swiglu_reference`
(reference.py:53-57). `cpu_reference_model` restates that on CPU tensors:
every projection's forward becomes `OracleQuantLinear.forward`, which runs the
oracle's dequantizer (oracle.quant, bit-exact with quant.py) and a torch CPU
matmul in the model dtype.
"""

from __future__ import annotations

import types

import numpy as np
import torch
import torch.nn as nn

from . import quant as oquant

_NP = {torch.float16: "float16", torch.bfloat16: "bfloat16"}


class OracleQuantLinear(nn.Module):
    """int4 linear computed the reference's dequantize-then-matmul way on CPU."""

    def __init__(self, packed: np.ndarray, scales: torch.Tensor, zeros: torch.Tensor, in_features: int,
                 out_features: int, bias: torch.Tensor | None, group_size: int) -> None:
        super().__init__()
        self.packed = packed
        self.scales = scales.float().numpy()
        self.zeros = zeros.float().numpy()
        self.bias = bias
        self.in_features = in_features
        self.out_features = out_features
        self.group_size = group_size

    @torch.no_grad()
    def forward(self, x: torch.Tensor) -> torch.Tensor:
        dense = oquant.dequantize_int4_f32(self.packed, self.scales, self.zeros, self.group_size)
        w = torch.from_numpy(dense[: self.in_features]).to(x.dtype)     # quant.py:105 (cast)
        shape = x.shape
        out = x.reshape(-1, shape[-1]) @ w                                # qwen.py:95
        if self.bias is not None:
            out = out + self.bias                                         # qwen.py:96-97
        return out.reshape(*shape[:-1], self.out_features)


def _swiglu_mlp_forward(self, x):
    g = self.gate_proj(x).float()
    u = self.up_proj(x).float()
    act = ((g * torch.sigmoid(g)) * u).to(x.dtype)                       # reference.py:53-57
    return self.down_proj(act)


def cpu_reference_model(cpu_model, patched_model) -> nn.Module:
    """Turn `cpu_model` (an unpatched transformers Qwen2 model on the CPU, same
    weights as `patched_model` before patching) into the reference's CPU path:
    its projections take the int4 buffers of `patched_model`'s QuantLinears
    (any device) and run dequantize-then-matmul. Modifies and returns cpu_model."""
    model = cpu_model.to("cpu")
    for layer, player in zip(model.model.layers, patched_model.model.layers):
        for parent, pparent, names in ((layer.self_attn, player.self_attn, ("q_proj", "k_proj", "v_proj", "o_proj")),
                                       (layer.mlp, player.mlp, ("gate_proj", "up_proj", "down_proj"))):
            for name in names:
                ql = getattr(pparent, name)
                setattr(parent, name, OracleQuantLinear(
                    ql.packed.cpu().numpy(), ql.scales.cpu(), ql.zeros.cpu(), ql.in_features,
                    ql.out_features, None if ql.bias is None else ql.bias.cpu(), ql.group_size))
        # norms stay transformers' RMSNorm; the MLP activation is the reference oracle
        layer.mlp.forward = types.MethodType(_swiglu_mlp_forward, layer.mlp)
    return model.eval()


def _rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    # transformers' Qwen2RMSNorm: fp32 variance, cast back, times the weight
    xf = x.float()
    xf = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return w * xf.to(x.dtype)


def _rotate(t: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    half = t.shape[-1] // 2
    rot = torch.cat((-t[..., half:], t[..., :half]), dim=-1)
    return t * cos + rot * sin


def random_int4_linear(n: int, k: int, gen: torch.Generator, dtype: torch.dtype, bias: bool = False,
                       group_size: int = 128):
    """An int4 linear [k -> n] in the reference's format with seeded random
    contents: codes uniform in 0..15 packed K-major (quant.py:25-63 layout),
    scales |N(0, 0.02)| x 4 / 15 (the range of N(0, 0.02) weights over 15
    steps), zeros uniform in 0..15, all on the host. For CPU timing samples,
    whose cost does not depend on the values; built without any GPU code."""
    k_pad = -(-k // group_size) * group_size
    packed = torch.randint(0, 256, (k_pad // 2, n), generator=gen, dtype=torch.uint8).numpy()
    scales = (torch.randn(k_pad // group_size, n, generator=gen).abs() * 0.02 * 4 / 15 + 1e-4).to(dtype)
    zeros = torch.randint(0, 16, (k_pad // group_size, n), generator=gen).to(dtype)
    b = (torch.randn(n, generator=gen) * 0.02).to(dtype) if bias else None
    return OracleQuantLinear(packed, scales, zeros, k, n, b, group_size)


def quantize_model_on_cpu(model: nn.Module, group_size: int = 128, dtype: torch.dtype = torch.float16) -> nn.Module:
    """The reference's patched model on the host: every q/k/v/o/gate/up/down
    Linear of a transformers Qwen2 model quantised by the oracle quantizer
    (bit-exact with quant.py:29-63) into an OracleQuantLinear, the MLP
    activation the SwiGLU oracle (integration/qwen.py:57-80 with
    fuse_max_m=0). Modifies and returns `model` (kept on the CPU)."""
    model = model.to("cpu")
    npdt = _NP[dtype]
    for layer in model.model.layers:
        for parent, names in ((layer.self_attn, ("q_proj", "k_proj", "v_proj", "o_proj")),
                              (layer.mlp, ("gate_proj", "up_proj", "down_proj"))):
            for name in names:
                lin = getattr(parent, name)
                packed, s_bits, z_bits, _ = oquant.quantize_int4_group(lin.weight.detach().float().numpy(),
                                                                       group_size, npdt)
                scales = torch.from_numpy(oquant.half_bits_to_f32(s_bits, npdt)).to(dtype)
                zeros = torch.from_numpy(oquant.half_bits_to_f32(z_bits, npdt)).to(dtype)
                bias = None if lin.bias is None else lin.bias.detach().to(dtype)
                setattr(parent, name, OracleQuantLinear(packed, scales, zeros, lin.in_features, lin.out_features,
                                                        bias, group_size))
        layer.mlp.forward = types.MethodType(_swiglu_mlp_forward, layer.mlp)
    return model.eval()


class CpuLayer:
    """One Qwen2 decoder layer of int4 weights on the CPU, computed the
    reference's way: dequantize-then-matmul projections (qwen.py:91-97),
    transformers' RMSNorm, rotary embedding and scaled-dot-product attention
    over the KV cache, the oracle SwiGLU (reference.py:53-57)."""

    def __init__(self, layer: dict, hidden: int, q_heads: int, kv_heads: int, head_dim: int, eps: float):
        def ql(q) -> OracleQuantLinear:
            if isinstance(q, OracleQuantLinear):
                return q
            return OracleQuantLinear(q.packed.cpu().numpy(), q.scales.cpu(), q.zeros.cpu(), q.in_features,
                                     q.out_features, None if q.bias is None else q.bias.cpu(), q.group_size)

        self.qkv, self.o, self.gu, self.down = ql(layer["qkv"]), ql(layer["o"]), ql(layer["gu"]), ql(layer["down"])
        self.in_norm, self.post_norm = layer["in_norm"].cpu(), layer["post_norm"].cpu()
        self.H, self.Hq, self.Hkv, self.D, self.eps = hidden, q_heads, kv_heads, head_dim, eps
        self.inter = self.gu.out_features // 2

    @torch.no_grad()
    def step(self, x: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, pos: int,
             cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
        """x [B, H] at position `pos`; caches [B, Hkv, T, D] hold positions < pos."""
        b = x.shape[0]
        h = _rms_norm(x, self.in_norm, self.eps)
        qkv = self.qkv(h)
        nq, nkv = self.Hq * self.D, self.Hkv * self.D
        q = qkv[:, :nq].view(b, self.Hq, 1, self.D)
        k = qkv[:, nq:nq + nkv].view(b, self.Hkv, 1, self.D)
        v = qkv[:, nq + nkv:].view(b, self.Hkv, 1, self.D)
        q, k = _rotate(q, cos[pos], sin[pos]), _rotate(k, cos[pos], sin[pos])
        k_cache[:, :, pos:pos + 1] = k
        v_cache[:, :, pos:pos + 1] = v
        g = self.Hq // self.Hkv
        kk = k_cache[:, :, :pos + 1].repeat_interleave(g, dim=1)
        vv = v_cache[:, :, :pos + 1].repeat_interleave(g, dim=1)
        attn = torch.nn.functional.scaled_dot_product_attention(q, kk, vv)
        attn = attn.reshape(b, nq)
        x = x + self.o(attn)
        h = _rms_norm(x, self.post_norm, self.eps)
        gu = self.gu(h).float()
        gate, up = gu[:, :self.inter], gu[:, self.inter:]
        act = ((gate * torch.sigmoid(gate)) * up).to(x.dtype)
        return x + self.down(act)

    @classmethod
    def random(cls, hidden: int, inter: int, q_heads: int, kv_heads: int, head_dim: int, eps: float,
               dtype: torch.dtype = torch.bfloat16, seed: int = 0) -> "CpuLayer":
        """A layer of the given shape with seeded random int4 contents
        (random_int4_linear: q|k|v with bias, gate|up concatenated), built on
        the host without any GPU code: the timing sample of a model too large
        for the CPU."""
        g = torch.Generator().manual_seed(seed)
        qkv = random_int4_linear((q_heads + 2 * kv_heads) * head_dim, hidden, g, dtype, bias=True)
        layer = {"qkv": qkv, "o": random_int4_linear(hidden, q_heads * head_dim, g, dtype),
                 "gu": random_int4_linear(2 * inter, hidden, g, dtype),
                 "down": random_int4_linear(hidden, inter, g, dtype),
                 "in_norm": torch.ones(hidden, dtype=dtype), "post_norm": torch.ones(hidden, dtype=dtype)}
        return cls(layer, hidden, q_heads, kv_heads, head_dim, eps)
