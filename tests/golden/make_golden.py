"""Generate golden vectors by running the reference implementation itself.

Run in a container where the reference checkout is importable::

    python tests/golden/make_golden.py /path/to/reference/src

It imports the reference's ``tritonforge.quant`` and ``tritonforge.reference``
(pure PyTorch, CPU) and records inputs and outputs for small seeded cases into
``tests/golden/kernels_golden.npz``. Half-precision tensors are stored as
``uint16`` bit patterns (``<name>__f16`` / ``<name>__bf16``). The tests never
import the reference; they read only this file.
"""

from __future__ import annotations

import pathlib
import sys

import numpy as np
import torch

OUT = pathlib.Path(__file__).resolve().parent / "kernels_golden.npz"


def _bits(t: torch.Tensor) -> tuple[str, np.ndarray]:
    if t.dtype == torch.float16:
        return "f16", t.contiguous().view(torch.int16).numpy().view(np.uint16)
    if t.dtype == torch.bfloat16:
        return "bf16", t.contiguous().view(torch.int16).numpy().view(np.uint16)
    if t.dtype == torch.float32:
        return "f32", t.contiguous().numpy()
    if t.dtype == torch.uint8:
        return "u8", t.contiguous().numpy()
    raise TypeError(t.dtype)


def main(ref_src: str) -> None:
    sys.path.insert(0, ref_src)
    from tritonforge import quant, reference  # the reference implementation

    rec: dict[str, np.ndarray] = {}

    def put(name: str, t: torch.Tensor) -> None:
        tag, arr = _bits(t)
        rec[f"{name}__{tag}"] = arr

    dt_name = {torch.float16: "f16", torch.bfloat16: "bf16"}

    # ---- quantizer / packer / dequantizer (quant.py) -------------------------
    quant_cases = [
        # (case, N, K, group, dtype, generator)
        ("layout_zero", 3, 8, 4, torch.float16, "zeros"),
        ("randn_64x256", 64, 256, 128, torch.float16, "randn"),
        ("pad_4x129", 4, 129, 128, torch.float16, "randn"),
        ("manual_8x128", 8, 128, 128, torch.float16, "randn"),
        ("bf16_37x300", 37, 300, 128, torch.bfloat16, "randn"),
        ("small_16x896", 16, 896, 128, torch.float16, "small"),
        ("bf16_g32_5x64", 5, 64, 32, torch.bfloat16, "randn"),
        ("edge_const", 6, 256, 128, torch.float16, "edge"),
        ("tiny_scale", 4, 256, 128, torch.float16, "tiny"),
    ]
    names = []
    for case, n, k, g, dt, gen in quant_cases:
        torch.manual_seed(len(names) + 11)
        if gen == "zeros":
            w = torch.zeros(n, k)
        elif gen == "randn":
            w = torch.randn(n, k)
        elif gen == "small":
            w = torch.randn(n, k) * 0.02
        elif gen == "tiny":
            w = torch.randn(n, k) * 1e-6
        else:  # constant rows, a zero row, mixed-sign constants, huge values
            w = torch.randn(n, k)
            w[0] = 1.0
            w[1] = -1.0
            w[2] = 0.0
            w[3, :128] = 3.5
            w[4] *= 1000.0
            w[5, 7] = 65000.0
        packed, scales, zeros, k_pad = quant.quantize_int4_group(w, g, dt)
        dense = quant.dequantize_int4(packed, scales, zeros, g, dt)
        codes = quant.unpack_int4(packed)
        p = f"quant/{case}"
        put(f"{p}/w", w)
        put(f"{p}/packed", packed)
        put(f"{p}/scales", scales)
        put(f"{p}/zeros", zeros)
        put(f"{p}/dense", dense)
        put(f"{p}/codes", codes)
        rec[f"{p}/meta"] = np.array([n, k, g, k_pad, 1 if dt == torch.bfloat16 else 0])
        names.append(case)
    rec["quant/cases"] = np.array(names)

    # known-answer pack test (reference tests/test_quant.py:12-18)
    q = torch.tensor([[0, 1, 2, 3, 4, 5, 6, 7], [8, 9, 10, 11, 12, 13, 14, 15]],
                     dtype=torch.uint8)
    packed = (q[:, 0::2].t().contiguous() | (q[:, 1::2].t().contiguous() << 4)).to(torch.uint8)
    put("kat/packed", packed)
    put("kat/codes", quant.unpack_int4(packed))

    # ---- quantized_linear_reference (reference.py:21-36) ---------------------
    lin_cases = [(1, 64, 128, True), (3, 127, 129, True), (16, 128, 256, True),
                 (17, 64, 256, True), (4, 32, 256, False), (2, 256, 384, True)]
    lnames = []
    for dt in (torch.float16, torch.bfloat16):
        for m, n, k, has_bias in lin_cases:
            torch.manual_seed(m * 1000 + n + k)
            x = torch.randn(m, k).to(dt)
            w = torch.randn(n, k)
            packed, scales, zeros, _ = quant.quantize_int4_group(w, 128, dt)
            bias = torch.randn(n).to(dt) if has_bias else None
            out = reference.quantized_linear_reference(x, packed, scales, zeros, bias, 128)
            p = f"linear/{dt_name[dt]}_{m}x{n}x{k}"
            put(f"{p}/x", x)
            put(f"{p}/packed", packed)
            put(f"{p}/scales", scales)
            put(f"{p}/zeros", zeros)
            if bias is not None:
                put(f"{p}/bias", bias)
            put(f"{p}/out", out)
            lnames.append(p)
    rec["linear/cases"] = np.array(lnames)

    # ---- rmsnorm_residual_reference (reference.py:39-50) ----------------------
    nnames = []
    for dt in (torch.float16, torch.bfloat16):
        for m, n in [(1, 896), (4, 896), (16, 1536), (3, 100)]:
            torch.manual_seed(m + n)
            x = torch.randn(m, n).to(dt)
            r = torch.randn(m, n).to(dt)
            w = torch.randn(n).to(dt)
            normed, summed = reference.rmsnorm_residual_reference(x, r, w, 1e-6)
            p = f"rmsnorm/{dt_name[dt]}_{m}x{n}"
            put(f"{p}/x", x)
            put(f"{p}/r", r)
            put(f"{p}/w", w)
            put(f"{p}/normed", normed)
            put(f"{p}/summed", summed)
            # plain RMSNorm, as the reference's integration test states it
            acc = x.to(torch.float32)
            var = acc.pow(2).mean(-1, keepdim=True)
            plain = (acc * torch.rsqrt(var + 1e-6)).to(dt) * w
            put(f"{p}/plain", plain)
            nnames.append(p)
    rec["rmsnorm/cases"] = np.array(nnames)

    # ---- swiglu_reference (reference.py:53-57) --------------------------------
    snames = []
    for dt in (torch.float16, torch.bfloat16):
        for shape in [(1, 4864), (3, 127), (16, 512)]:
            torch.manual_seed(shape[0] * 7 + shape[1])
            g = (torch.randn(*shape) * 4).to(dt)
            u = torch.randn(*shape).to(dt)
            out = reference.swiglu_reference(g, u)
            p = f"swiglu/{dt_name[dt]}_{shape[0]}x{shape[1]}"
            put(f"{p}/g", g)
            put(f"{p}/u", u)
            put(f"{p}/out", out)
            snames.append(p)
    rec["swiglu/cases"] = np.array(snames)

    np.savez_compressed(OUT, **rec)
    print(f"wrote {OUT} ({OUT.stat().st_size / 1024:.1f} KiB, {len(rec)} arrays)")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit(f"usage: python {sys.argv[0]} <path to the reference's src directory>")
    main(sys.argv[1])
