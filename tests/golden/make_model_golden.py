"""Greedy-decode golden tokens for the Qwen2.5-0.5B-shaped model, produced by
the reference implementation on the CPU.

    python tests/golden/make_model_golden.py /path/to/reference/src

Model: transformers Qwen2ForCausalLM with the Qwen2.5-0.5B shape, random init
under torch.manual_seed(0), fp16 (tritonforge_b200.decode.random_qwen2).
Oracle: the reference's own `patch_model(model, fuse_max_m=0, fuse_norm=False,
fuse_mlp=False)` -- every q/k/v/o/gate/up/down becomes the reference's int4
QuantLinear running its dequantize-then-matmul path, norms stay transformers'
RMSNorm (the oracle's two-rounding form) -- with each MLP's activation computed
by the reference's `swiglu_reference` (reference.py:53-57), i.e. the reference
patched model with its fused kernels replaced by their reference.py oracles.
Prompts are uniform random token ids (seeded); 32 greedy steps are recorded
with the top-1/top-2 logit gap of every step.
"""

from __future__ import annotations

import pathlib
import sys
import time
import types

import numpy as np
import torch

ROOT = pathlib.Path(__file__).resolve().parents[2]
OUT = pathlib.Path(__file__).resolve().parent / "qwen05b_greedy.npz"
PROMPT_LEN, NEW_TOKENS, BATCH = 128, 32, 2


def weight_checksum(model) -> np.ndarray:
    sd = model.state_dict()
    keys = ["model.embed_tokens.weight", "model.layers.0.self_attn.q_proj.weight",
            "model.layers.23.mlp.down_proj.weight", "model.norm.weight"]
    return np.array([sd[k].double().sum().item() for k in keys])


def main(ref_src: str) -> None:
    sys.path.insert(0, str(ROOT))
    from tritonforge_b200.decode import random_qwen2

    model = random_qwen2("0.5b", seed=0)
    checksum = weight_checksum(model)
    sys.path.insert(0, ref_src)
    from tritonforge import reference
    from tritonforge.integration import patch_model

    patch_model(model, group_size=128, fuse_max_m=0, dtype=torch.float16,
                quantize=True, fuse_norm=False, fuse_mlp=False)

    def mlp_forward(self, x):
        return self.down_proj(reference.swiglu_reference(self.gate_proj(x), self.up_proj(x)))

    for layer in model.model.layers:
        layer.mlp.forward = types.MethodType(mlp_forward, layer.mlp)

    g = torch.Generator().manual_seed(1234)
    prompt = torch.randint(0, model.config.vocab_size, (BATCH, PROMPT_LEN), generator=g)
    torch.set_num_threads(max(1, torch.get_num_threads()))
    t0 = time.time()
    tokens, gaps = [], []
    with torch.no_grad():
        out = model(prompt, use_cache=True)
        for step in range(NEW_TOKENS):
            logits = out.logits[:, -1, :].float()
            top2 = logits.topk(2, dim=-1).values
            gaps.append((top2[:, 0] - top2[:, 1]).numpy())
            nxt = logits.argmax(-1, keepdim=True)
            tokens.append(nxt[:, 0].numpy())
            if step + 1 < NEW_TOKENS:
                out = model(nxt, past_key_values=out.past_key_values, use_cache=True)
    tokens = np.stack(tokens, axis=1)
    gaps = np.stack(gaps, axis=1)
    np.savez_compressed(OUT, prompt=prompt.numpy(), tokens=tokens, top2_gap=gaps, checksum=checksum)
    print(f"wrote {OUT} in {time.time() - t0:.0f}s; tokens[0][:8]={tokens[0][:8]}, "
          f"min top-2 gap {gaps.min():.4f}")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit(f"usage: python {sys.argv[0]} <path to the reference's src directory>")
    main(sys.argv[1])
