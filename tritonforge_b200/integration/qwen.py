"""Qwen2 integration: run a transformers ``Qwen2ForCausalLM`` on the B200 kernels.

Public surface kept from the reference (src/tritonforge/integration/qwen.py):
``QuantLinear(packed, scales, zeros, in_features, out_features, bias=None,
group_size=128, fuse_max_m=128)`` with its ``from_linear`` constructor and
buffers ``packed/scales/zeros/bias`` (:30-98), and ``patch_model(model,
group_size=128, fuse_max_m=128, dtype=fp16, quantize=True, fuse_norm=True,
fuse_mlp=True)`` (:155-185). How the patched model runs is this package's own:

* ``QuantLinear`` sends every M to ``kernels.quantized_linear``, whose native
  dispatcher picks the decode GEMV, the tcgen05 GEMM or the generic kernel
  (the reference hands M > ``fuse_max_m`` to dequantise-then-cuBLAS; the
  attribute is kept for compatibility).
* ``fuse_norm``: layer boundaries become one ``rmsnorm_residual`` launch each.
  A patched layer ends by adding its MLP output to the residual stream *and*
  normalising the sum with the norm that reads it next (the following layer's
  input norm, or the model's final norm) in the same kernel; it returns the
  sum, as transformers expects, and leaves the normalised copy in a per-model
  ``_Handoff`` that the next norm returns instead of recomputing. The first
  layer's input norm is a plain ``rmsnorm``; the post-attention norm is
  ``rmsnorm_residual``. Values are the reference's: ``summed = round(h + r)``
  and the norm of the rounded sum with the same roundings.
* ``fuse_mlp``: with int4 projections, gate and up live in one interleaved
  ``QuantLinear`` (columns [gate 64 | up 64] per 128) and up to 32 rows run the
  fused gate|up + SwiGLU decode kernel (``tf_qlinear_swiglu``: one launch, no
  [M, 2I] round trip); longer inputs run the two projections and ``swiglu``.
  Unquantised projections get ``swiglu`` between them.
"""

from __future__ import annotations

import torch
import torch.nn as nn

from .. import _lib, kernels, quant

DEFAULT_FUSE_MAX_M = 128
_FUSED_GATE_UP_MAX_M = 32  # rows the fused gate|up + SwiGLU decode kernel serves


def _rows(x: torch.Tensor) -> torch.Tensor:
    """x viewed as [rows, features] (a copy only when the layout requires it)."""
    return x.reshape(-1, x.shape[-1])


class QuantLinear(nn.Module):
    """A linear layer whose weight is int4, group-quantised along K and packed
    K-major (``packed [K_pad/2, N]`` uint8, ``scales``/``zeros [K_pad/g, N]``):
    the reference's format (quant.py:25-63). ``fuse_max_m`` is kept for
    signature compatibility; the native dispatcher picks the kernel by M."""

    def __init__(self, packed: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor, in_features: int,
                 out_features: int, bias: torch.Tensor | None = None, group_size: int = 128,
                 fuse_max_m: int = DEFAULT_FUSE_MAX_M) -> None:
        super().__init__()
        self.in_features, self.out_features = int(in_features), int(out_features)
        self.group_size, self.fuse_max_m = int(group_size), int(fuse_max_m)
        for name, t in (("packed", packed), ("scales", scales), ("zeros", zeros)):
            self.register_buffer(name, t)
        self.register_buffer("bias", bias)

    @classmethod
    def from_linear(cls, linear: nn.Linear, group_size: int = 128, dtype: torch.dtype = torch.float16,
                    fuse_max_m: int = DEFAULT_FUSE_MAX_M) -> "QuantLinear":
        """Quantise an ``nn.Linear`` where its weight lives (the CUDA quantizer
        on a GPU; quant.py:29-63 semantics, bit for bit), bias cast to ``dtype``."""
        w = linear.weight.detach()
        packed, scales, zeros, _ = quant.quantize_int4_group(w.float(), group_size, dtype)
        dev = w.device
        bias = None if linear.bias is None else linear.bias.detach().to(device=dev, dtype=dtype).contiguous()
        return cls(packed.to(dev), scales.to(dev), zeros.to(dev), linear.in_features, linear.out_features, bias,
                   group_size, fuse_max_m)

    def extra_repr(self) -> str:
        return (f"in_features={self.in_features}, out_features={self.out_features}, int4 group "
                f"{self.group_size}, bias={self.bias is not None}")

    @torch.no_grad()
    def forward(self, x: torch.Tensor) -> torch.Tensor:
        y = kernels.quantized_linear(_rows(x), self.packed, self.scales, self.zeros, self.bias, self.group_size)
        return y.view(*x.shape[:-1], self.out_features)


def _interleaved_gate_up(gate: QuantLinear, up: QuantLinear) -> QuantLinear | None:
    """gate and up as one QuantLinear with columns [gate 64 | up 64] per 128
    (the fused gate|up + SwiGLU kernel's layout), or None when the pair does
    not fit that kernel (a bias, or an intermediate width not a multiple of 64)."""
    from ..tp import interleave_gate_up

    if gate.bias is not None or up.bias is not None or gate.out_features % 64 or gate.packed.shape != up.packed.shape:
        return None
    return QuantLinear(interleave_gate_up(gate.packed, up.packed).contiguous(),
                       interleave_gate_up(gate.scales, up.scales).contiguous(),
                       interleave_gate_up(gate.zeros, up.zeros).contiguous(),
                       gate.in_features, 2 * gate.out_features, None, gate.group_size, gate.fuse_max_m)


class _SwiGLUMLP(nn.Module):
    """``down(silu(gate(x)) * up(x))`` on the native kernels. Keeps the
    module's ``gate_proj``/``up_proj``/``down_proj`` (and their attributes);
    int4 gate/up also get an interleaved copy for the fused decode kernel."""

    def __init__(self, mlp: nn.Module) -> None:
        super().__init__()
        self.gate_proj, self.up_proj, self.down_proj = mlp.gate_proj, mlp.up_proj, mlp.down_proj
        self.gate_up = None
        if isinstance(self.gate_proj, QuantLinear) and isinstance(self.up_proj, QuantLinear):
            self.gate_up = _interleaved_gate_up(self.gate_proj, self.up_proj)

    @torch.no_grad()
    def forward(self, x: torch.Tensor) -> torch.Tensor:
        x2 = _rows(x)
        gu = self.gate_up
        if gu is not None and 0 < x2.shape[0] <= _FUSED_GATE_UP_MAX_M and x2.is_cuda:
            act = self._fused_gate_up(x2.contiguous(), gu)
            if act is not None:
                return self.down_proj(act).view(*x.shape[:-1], -1)
        act = kernels.swiglu(self.gate_proj(x2), self.up_proj(x2))
        return self.down_proj(act).view(*x.shape[:-1], -1)

    @staticmethod
    def _fused_gate_up(x2: torch.Tensor, gu: QuantLinear) -> torch.Tensor | None:
        m, k = x2.shape
        lib = _lib.load()
        act = torch.empty(m, gu.out_features // 2, dtype=x2.dtype, device=x2.device)
        ws = _lib.workspaces.get(x2.device, 256)
        rc = lib.tf_qlinear_swiglu(x2.data_ptr(), x2.stride(0), _lib.dtype_code(x2.dtype), gu.packed.data_ptr(),
                                   gu.scales.data_ptr(), gu.zeros.data_ptr(), _lib.dtype_code(gu.scales.dtype),
                                   act.data_ptr(), act.stride(0), m, gu.out_features, k, gu.packed.shape[0] * 2,
                                   gu.group_size, ws.data_ptr(), ws.numel(), _lib.stream_ptr(x2.device))
        if rc == _lib.ERR_UNSUPPORTED:
            return None  # a shape or alignment the decode kernel does not take: run the two projections
        _lib.check(rc, "qlinear_swiglu")
        return act


class _Handoff:
    """The normalised copy of the hidden state a patched layer returned
    (computed in the same kernel as the residual add), waiting for the norm
    that consumes it. Identity of the returned tensor ties the two together:
    a norm handed any other tensor normalises it itself."""

    def __init__(self) -> None:
        self.summed: torch.Tensor | None = None
        self.normed: torch.Tensor | None = None

    def take(self, hidden: torch.Tensor) -> torch.Tensor | None:
        if self.summed is not None and hidden is self.summed:
            normed, self.summed, self.normed = self.normed, None, None
            return normed
        return None


class _BoundaryNorm(nn.Module):
    """An RMSNorm (input norm of a layer, or the model's final norm) that
    returns the handed-off normalised state when it is given the tensor the
    previous patched layer returned, and runs ``kernels.rmsnorm`` otherwise.
    Keeps the wrapped norm's ``weight`` and ``variance_epsilon``."""

    def __init__(self, norm: nn.Module, handoff: _Handoff) -> None:
        super().__init__()
        self.weight = norm.weight
        self.variance_epsilon = float(getattr(norm, "variance_epsilon", getattr(norm, "eps", 1e-6)))
        self._handoff = handoff

    @torch.no_grad()
    def forward(self, hidden: torch.Tensor) -> torch.Tensor:
        ready = self._handoff.take(hidden)
        if ready is not None:
            return ready
        return kernels.rmsnorm(_rows(hidden), self.weight, self.variance_epsilon).view(hidden.shape)


class _FusedBoundaryLayer(nn.Module):
    """A Qwen2 decoder layer whose two residual adds are fused with the norm
    that follows each: after attention with its own post-attention norm, after
    the MLP with `next_norm` (the next layer's input norm or the final norm),
    whose result goes to the handoff. Holds the original layer's submodules;
    returns a Tensor (the transformers 5.x decoder-layer contract)."""

    def __init__(self, layer: nn.Module, handoff: _Handoff) -> None:
        super().__init__()
        self.self_attn, self.mlp = layer.self_attn, layer.mlp
        self.input_layernorm = _BoundaryNorm(layer.input_layernorm, handoff)
        self.post_attention_layernorm = layer.post_attention_layernorm
        self.attention_type = getattr(layer, "attention_type", "full_attention")
        # the norm that reads this layer's output, set by patch_model once every
        # layer is wrapped; kept in a tuple so it is not registered as a child
        self._next: tuple = ()
        self._handoff = handoff

    def forward(self, hidden_states: torch.Tensor, *args, **kwargs) -> torch.Tensor:
        h = self.input_layernorm(hidden_states)
        attn = self.self_attn(h, *args, **kwargs)
        attn = attn[0] if isinstance(attn, tuple) else attn
        shape = hidden_states.shape
        post = self.post_attention_layernorm
        normed, stream = kernels.rmsnorm_residual(_rows(attn), _rows(hidden_states), post.weight,
                                                  post.variance_epsilon)
        out = _rows(self.mlp(normed.view(shape)))
        if not self._next:
            return (stream + out).view(shape)
        nxt = self._next[0]
        normed_next, summed = kernels.rmsnorm_residual(out, stream, nxt.weight, nxt.variance_epsilon)
        summed = summed.view(shape)
        self._handoff.summed, self._handoff.normed = summed, normed_next.view(shape)
        return summed


def patch_model(model: nn.Module, group_size: int = 128, fuse_max_m: int = DEFAULT_FUSE_MAX_M,
                dtype: torch.dtype = torch.float16, quantize: bool = True, fuse_norm: bool = True,
                fuse_mlp: bool = True) -> nn.Module:
    """Patch a transformers Qwen2 model in place and return it: ``quantize``
    turns the seven projections of every layer into int4 ``QuantLinear``s,
    ``fuse_mlp`` runs each MLP as ``_SwiGLUMLP``, ``fuse_norm`` wraps each
    decoder layer so its residual adds are fused with the following norms."""
    inner = model.model
    projections = (("self_attn", ("q_proj", "k_proj", "v_proj", "o_proj")),
                   ("mlp", ("gate_proj", "up_proj", "down_proj")))
    for layer in inner.layers:
        if quantize:
            for part, names in projections:
                parent = getattr(layer, part)
                for name in names:
                    lin = getattr(parent, name, None)
                    if isinstance(lin, nn.Linear):
                        setattr(parent, name, QuantLinear.from_linear(lin, group_size, dtype, fuse_max_m))
        if fuse_mlp and not isinstance(layer.mlp, _SwiGLUMLP):
            layer.mlp = _SwiGLUMLP(layer.mlp)
    if fuse_norm:
        handoff = _Handoff()
        wrapped = [l if isinstance(l, _FusedBoundaryLayer) else _FusedBoundaryLayer(l, handoff) for l in inner.layers]
        for i, l in enumerate(wrapped):
            inner.layers[i] = l
        if not isinstance(inner.norm, _BoundaryNorm):
            inner.norm = _BoundaryNorm(inner.norm, handoff)
        for l, nxt in zip(wrapped, wrapped[1:] + [None]):
            l._next = (nxt.input_layernorm if nxt is not None else inner.norm,)
    return model
