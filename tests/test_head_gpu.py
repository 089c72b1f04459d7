"""GPU tests of the decode step's head: tf_embed_gather (exact), and
tf_lm_head_argmax (logits within the contract of a float64 product, the
greedy token equal to torch.argmax over the kernel's own rounded logits, ties
to the smallest id across CTAs, the (logit, id) pairs of vocabulary slices
combined by tf_best_of_ranks, the position counters advanced)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from tests.parity import assert_rms_close, f32
from tritonforge_b200 import _lib

pytestmark = pytest.mark.gpu


def _ws(nbytes: int) -> torch.Tensor:
    return torch.zeros(nbytes, dtype=torch.uint8, device="cuda")


def _head(x, w, logits=None, tokens=None, best=None, v0=0, pos=None, ws=None):
    lib = _lib.load()
    B, H = x.shape
    V = w.shape[0]
    ws = ws if ws is not None else _ws(lib.tf_lm_head_workspace_bytes(B))
    rc = lib.tf_lm_head_argmax(x.data_ptr(), x.stride(0), w.data_ptr(), w.stride(0), V, H, B, _lib.dtype_code(x.dtype),
                               logits.data_ptr() if logits is not None else None,
                               logits.stride(0) if logits is not None else 0,
                               tokens.data_ptr() if tokens is not None else None,
                               best.data_ptr() if best is not None else None, v0,
                               pos.data_ptr() if pos is not None else None, pos.numel() if pos is not None else 0,
                               ws.data_ptr(), ws.numel(), _lib.stream_ptr(x.device))
    _lib.check(rc, "lm_head_argmax")
    return ws


def test_embed_gather_exact():
    lib = _lib.load()
    g = torch.Generator().manual_seed(0)
    V, H, B = 1000, 896, 6
    embed = torch.randn(V, H, generator=g).to(torch.bfloat16).cuda()
    tokens = torch.tensor([3, 999, 0, 3, -1, 1000], dtype=torch.long, device="cuda")
    x = torch.full((B, H), float("nan"), dtype=torch.bfloat16, device="cuda")
    res = torch.full((B, H + 64), float("nan"), dtype=torch.bfloat16, device="cuda")
    _lib.check(lib.tf_embed_gather(embed.data_ptr(), embed.stride(0), tokens.data_ptr(), x.data_ptr(), x.stride(0),
                                   res.data_ptr(), res.stride(0), V, H, B, _lib.BF16, _lib.stream_ptr(x.device)),
               "embed_gather")
    torch.cuda.synchronize()
    for b, t in enumerate(tokens.tolist()):
        want = embed[t] if 0 <= t < V else torch.zeros(H, dtype=torch.bfloat16, device="cuda")
        assert torch.equal(x[b], want) and torch.equal(res[b, :H], want)
    assert torch.isnan(res[:, H:].float()).all(), "no write beyond H"


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("B,V,H", [(1, 5000, 896), (7, 12345, 1024), (32, 30000, 3584), (64, 4096, 2048),
                                   (17, 152064, 256), (2, 37, 8192)])
def test_lm_head_argmax(B, V, H, dtype):
    g = torch.Generator().manual_seed(B + V + H)
    x = torch.randn(B, H, generator=g).to(dtype).cuda()
    w = (torch.randn(V, H, generator=g) * 0.02).to(dtype).cuda()
    logits = torch.full((B, V), float("nan"), dtype=dtype, device="cuda")
    tokens = torch.full((B,), -7, dtype=torch.long, device="cuda")
    pos = torch.tensor([41, 42], dtype=torch.int32, device="cuda")
    ws = _head(x, w, logits=logits, tokens=tokens, pos=pos)
    torch.cuda.synchronize()
    ref = f32(x).astype(np.float64) @ f32(w).astype(np.float64).T
    assert_rms_close(logits, ref, dtype, f"lm_head {B}x{V}x{H}")
    # the greedy token is the first maximum of the kernel's own rounded logits ...
    assert torch.equal(tokens, torch.argmax(logits, dim=-1))
    # ... which is a true maximum up to the rounding of the logits
    top = ref.max(axis=1)
    picked = ref[np.arange(B), tokens.cpu().numpy()]
    ulp = np.ldexp(1.0, np.frexp(np.abs(top))[1] - (8 if dtype == torch.bfloat16 else 11))
    assert (picked >= top - 2 * ulp).all()
    assert pos.tolist() == [42, 43]
    assert int(ws[:4].view(torch.int32).item()) == 0, "a bounded wait expired"
    # the counter is left zeroed: a second call on the same workspace agrees
    tokens2 = torch.empty_like(tokens)
    _head(x, w, tokens=tokens2, ws=ws)
    torch.cuda.synchronize()
    assert torch.equal(tokens2, tokens)


def test_lm_head_ties_go_to_the_smallest_id():
    """Rows 7 and 3000 (different CTAs) and 11 give the same largest logit:
    the smallest id wins, as with torch.argmax."""
    H, V = 1024, 5000
    g = torch.Generator().manual_seed(3)
    v = torch.randn(H, generator=g).abs().to(torch.bfloat16)
    w = torch.zeros(V, H, dtype=torch.bfloat16)
    for r in (3000, 11, 7):
        w[r] = v
    x = v.unsqueeze(0).repeat(3, 1).cuda()
    x[1] *= -1  # every logit but rows 7, 11, 3000 is 0 and those are negative: row 0 wins
    tokens = torch.empty(3, dtype=torch.long, device="cuda")
    _head(x, w.cuda(), tokens=tokens)
    torch.cuda.synchronize()
    assert tokens.tolist() == [7, 0, 7]


def test_lm_head_vocab_slices_and_best_of_ranks():
    """Each rank's slice gives (best logit, global id); tf_best_of_ranks picks
    the token torch.argmax finds over the whole vocabulary."""
    lib = _lib.load()
    B, V, H, world = 5, 9000, 2048, 3
    g = torch.Generator().manual_seed(11)
    x = torch.randn(B, H, generator=g).to(torch.bfloat16).cuda()
    w = (torch.randn(V, H, generator=g) * 0.02).to(torch.bfloat16).cuda()
    full = torch.empty(B, V, dtype=torch.bfloat16, device="cuda")
    _head(x, w, logits=full)
    edges = [0, 2999, 6000, V]
    all_best = torch.empty(world, B, 2, dtype=torch.float32, device="cuda")
    for r in range(world):
        sl = w[edges[r]:edges[r + 1]].contiguous()
        _head(x, sl, best=all_best[r], v0=edges[r])
    tokens = torch.empty(B, dtype=torch.long, device="cuda")
    _lib.check(lib.tf_best_of_ranks(all_best.data_ptr(), tokens.data_ptr(), world, B, _lib.stream_ptr(x.device)),
               "best_of_ranks")
    torch.cuda.synchronize()
    assert torch.equal(tokens, torch.argmax(full, dim=-1))


def test_engine_head_above_64_rows():
    """A decode step at batch 100 runs the lm_head + argmax as two launches
    (64 + 36 rows): every row's logits against torch's fp32 product of the
    step's final normed rows, every token a maximum of its row, and the
    position advanced once."""
    from tritonforge_b200.decode import QwenDecoder, QwenWeights

    dev = torch.device("cuda", 0)
    w = QwenWeights.synthetic("7b", dtype=torch.bfloat16, device=dev, seed=5, layers=1)
    d = QwenDecoder(w, 100, 32, colmajor=False)
    d.fill_cache(8, seed=2)
    pos0 = d.pos.clone()
    d.step()
    torch.cuda.synchronize()
    assert (d.pos - pos0).tolist() == [1, 1]
    logits = d.buf["logits"].float()
    want = d.buf["normed"].float() @ w.lm_head.float().T
    rms = float(want.pow(2).mean().sqrt())
    assert float((logits - want).abs().max()) <= 2e-2 * rms
    assert torch.equal(logits.gather(1, d.tokens[:, None])[:, 0], logits.max(-1).values)
    assert d.device_errors() == 0
