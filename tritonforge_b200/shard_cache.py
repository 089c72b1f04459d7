"""On-disk cache of one rank's quantised decoder weights.

Quantising a 72B model (reference src/tritonforge/quant.py:29-63, about 70 B
parameters) takes far longer than loading its result, so a run can save the
int4 shards it produced once and load them on later runs. The tensors are
stored in the reference's own formats — packed uint8 [K_pad/2, N] K-major,
scales and zeros [K_pad/g, N], bias [N] — one rank's tensor-parallel shard
per directory:

    <dir>/manifest.json   format tag, decoder shape, tensor-parallel degree
                          and rank, the layout of the fused projections,
                          the size of tensors.bin, tensor table
    <dir>/tensors.bin     the tensors' raw little-endian bytes, each at a
                          256-byte-aligned offset

Both files are written under temporary names and renamed (blob first); the
manifest records the blob's size, so a blob that does not belong to its
manifest (an interrupted save) fails the load instead of loading.

Raw bytes plus a JSON table keep the files readable without Python (a host
runtime can memory-map tensors.bin and take offsets from the manifest). A
load returns the same bits that were saved.
"""

from __future__ import annotations

import json
import os

import numpy as np
import torch

FORMAT = "tritonforge_b200-int4-shard/2"
# how the decoder's fused projections are laid out (checked on load)
LAYOUT = {"qkv": "q|k|v projections concatenated along N (q heads, then k, then v)",
          "gu": "gate|up interleaved per 64 columns: [gate 0:64 | up 0:64 | gate 64:128 | ...]"}
_ALIGN = 256
_DTYPES = {torch.uint8: ("u8", np.uint8), torch.float16: ("f16", np.uint16), torch.bfloat16: ("bf16", np.uint16),
           torch.float32: ("f32", np.float32), torch.int32: ("i32", np.int32)}
_BY_TAG = {tag: (dt, npdt) for dt, (tag, npdt) in _DTYPES.items()}
_LINEARS = ("qkv", "o", "gu", "down")
_FIELDS = ("hidden", "inter", "q_heads", "kv_heads", "head_dim", "eps", "rope_theta")


def _to_bytes(t: torch.Tensor) -> bytes:
    tag, npdt = _DTYPES[t.dtype]
    a = t.detach().contiguous().cpu()
    if t.dtype in (torch.float16, torch.bfloat16):
        a = a.view(torch.int16)
    return a.numpy().view(npdt).tobytes()


def save_weights(w, path: str, tp: int = 1, rank: int = 0) -> None:
    """Write `w` (rank `rank` of a `tp`-way tensor-parallel shard, as a
    QwenWeights whose projections are K-major QuantLinear) to the directory
    `path` (created if needed; existing files are replaced)."""
    from .integration.qwen import QuantLinear

    os.makedirs(path, exist_ok=True)
    table: dict[str, dict] = {}
    linears: dict[str, dict] = {}
    tmp = os.path.join(path, "tensors.bin.tmp")
    with open(tmp, "wb") as f:
        def put(name: str, t: torch.Tensor) -> None:
            pad = (-f.tell()) % _ALIGN
            if pad:
                f.write(b"\0" * pad)
            table[name] = {"dtype": _DTYPES[t.dtype][0], "shape": list(t.shape), "offset": f.tell()}
            f.write(_to_bytes(t))

        for li, L in enumerate(w.layers):
            put(f"layers.{li}.in_norm", L["in_norm"])
            put(f"layers.{li}.post_norm", L["post_norm"])
            for n in _LINEARS:
                ql = L[n]
                if not isinstance(ql, QuantLinear):
                    raise TypeError(f"layer {li} {n}: only K-major QuantLinear projections are saved "
                                    "(save before converting to the column-major layout)")
                p = f"layers.{li}.{n}"
                put(p + ".packed", ql.packed)
                put(p + ".scales", ql.scales)
                put(p + ".zeros", ql.zeros)
                if ql.bias is not None:
                    put(p + ".bias", ql.bias)
                linears[p] = {"in_features": ql.in_features, "out_features": ql.out_features,
                              "group_size": ql.group_size}
        put("embed", w.embed)
        tied = w.lm_head is w.embed or (w.lm_head.data_ptr() == w.embed.data_ptr() and
                                        w.lm_head.shape == w.embed.shape)
        if not tied:
            put("lm_head", w.lm_head)
        put("final_norm", w.final_norm)
    manifest = {"format": FORMAT, "tp": int(tp), "rank": int(rank), "layout": LAYOUT,
                "blob_bytes": os.path.getsize(tmp), "layers": len(w.layers), "tied_lm_head": bool(tied),
                "config": {k: getattr(w, k) for k in _FIELDS}, "linears": linears, "tensors": table}
    mtmp = os.path.join(path, "manifest.json.tmp")
    with open(mtmp, "w") as f:
        json.dump(manifest, f, indent=1)
    os.replace(tmp, os.path.join(path, "tensors.bin"))
    os.replace(mtmp, os.path.join(path, "manifest.json"))


def load_weights(path: str, device=None, tp: int | None = None, rank: int | None = None):
    """Read a directory written by `save_weights` into a QwenWeights on
    `device` (default: the current CUDA device). Raises ValueError for a
    directory of another format or layout, a blob that does not match its
    manifest, truncated data, or a shard of another tensor-parallel degree or
    rank than `tp` / `rank` (when given)."""
    from .decode import QwenWeights
    from .integration.qwen import QuantLinear

    with open(os.path.join(path, "manifest.json")) as f:
        man = json.load(f)
    if man.get("format") != FORMAT:
        raise ValueError(f"{path}: not a {FORMAT} directory (format {man.get('format')!r})")
    if man.get("layout") != LAYOUT:
        raise ValueError(f"{path}: fused projections in another layout: {man.get('layout')!r}")
    if tp is not None and man.get("tp") != tp or rank is not None and man.get("rank") != rank:
        raise ValueError(f"{path}: shard of tp={man.get('tp')} rank={man.get('rank')}, wanted tp={tp} rank={rank}")
    if os.path.getsize(os.path.join(path, "tensors.bin")) != man.get("blob_bytes"):
        raise ValueError(f"{path}: tensors.bin does not match its manifest (size differs)")
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device())
    blob = np.memmap(os.path.join(path, "tensors.bin"), dtype=np.uint8, mode="r")

    def get(name: str) -> torch.Tensor:
        e = man["tensors"][name]
        dt, npdt = _BY_TAG[e["dtype"]]
        count = int(np.prod(e["shape"])) if e["shape"] else 1
        nbytes = count * np.dtype(npdt).itemsize
        if e["offset"] + nbytes > blob.size:
            raise ValueError(f"{path}: tensor {name} runs past the end of tensors.bin")
        a = np.frombuffer(blob, dtype=npdt, count=count, offset=e["offset"]).reshape(e["shape"])
        t = torch.from_numpy(a.copy())
        if dt in (torch.float16, torch.bfloat16):
            t = t.view(torch.int16).view(dt)
        return t.to(device)

    layers = []
    for li in range(man["layers"]):
        L = {"in_norm": get(f"layers.{li}.in_norm"), "post_norm": get(f"layers.{li}.post_norm")}
        for n in _LINEARS:
            p = f"layers.{li}.{n}"
            meta = man["linears"][p]
            bias = get(p + ".bias") if p + ".bias" in man["tensors"] else None
            L[n] = QuantLinear(get(p + ".packed"), get(p + ".scales"), get(p + ".zeros"), meta["in_features"],
                               meta["out_features"], bias, meta["group_size"])
        layers.append(L)
    embed = get("embed")
    lm_head = embed if man["tied_lm_head"] else get("lm_head")
    c = man["config"]
    return QwenWeights(layers, embed, lm_head, get("final_norm"), c["hidden"], c["inter"], c["q_heads"],
                       c["kv_heads"], c["head_dim"], c["eps"], c["rope_theta"])
