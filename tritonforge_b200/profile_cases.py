"""One kernel of the decode / prefill path on a bounded case, for an ncu
capture of a single launch (the first launches are warm-up):

    python -m tritonforge_b200.profile_cases gemv|gemv_cm|attention|gemm

gemv:      int4 GEMV of the Qwen2.5-72B gate|up projection (K=8192, N=59136,
           bf16, int4 g128) at M=32 rows (the 72B decode at batch 32);
           242 MB of packed weights, larger than the 126 MB L2.
gemv_cm:   the same projection with the weights in the tiled column-major
           layout (tcgen05 decode kernel, tf_qlinear_cm).
attention: decode attention of the 72B shape (64 q / 8 kv heads of 128) at
           batch 32 over a 4096-position bf16 KV cache (1.07 GB of K/V).
gemm:      prefill-regime int4 linear of the 7B gate projection (K=3584,
           N=18944) at M=2048 rows, bf16.
"""

import sys

import torch

from tritonforge_b200 import _lib, colmajor, kernels, quant


def main(case: str) -> None:
    dt = torch.bfloat16
    if case in ("gemv", "gemm"):
        m, k, n = (32, 8192, 59136) if case == "gemv" else (2048, 3584, 18944)
        w = torch.randn(n, k, device="cuda") * 0.02
        p, s, z, _ = quant.quantize_int4_group(w, 128, dt)
        del w
        x = torch.randn(m, k, device="cuda").to(dt)
        out = torch.empty(m, n, device="cuda", dtype=dt)
        for _ in range(3):
            kernels.quantized_linear(x, p, s, z, None, 128, {"regime": case}, out=out)
    elif case == "gemv_cm":
        m, k, n = 32, 8192, 59136
        w = torch.randn(n, k, device="cuda") * 0.02
        p, s, z, _ = quant.quantize_int4_group(w, 128, dt)
        del w
        tiles = colmajor.repack_cm(p)
        del p
        x = torch.randn(m, k, device="cuda").to(dt)
        out = torch.empty(m, n, device="cuda", dtype=dt)
        for _ in range(3):
            colmajor.quantized_linear_cm(x, tiles, s, z, None, 128, out=out)
    elif case == "attention":
        b, hq, hkv, d, ctx = 32, 64, 8, 128, 4096
        t_max = ctx + 64
        kc = torch.randn(b, hkv, t_max, d, device="cuda", dtype=dt)
        vc = torch.randn(b, hkv, t_max, d, device="cuda", dtype=dt)
        q = torch.randn(b, hq, d, device="cuda", dtype=dt)
        out = torch.empty(b, hq * d, device="cuda", dtype=dt)
        lens = torch.tensor([ctx, ctx + 1], dtype=torch.int32, device="cuda")
        lib = _lib.load()
        for _ in range(3):
            _lib.check(lib.tf_decode_attention(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), out.data_ptr(),
                                               lens.data_ptr() + 4, b, hq, hkv, d, t_max, d ** -0.5,
                                               _lib.dtype_code(dt), _lib.stream_ptr(q.device)), "decode_attention")
    else:
        raise SystemExit(f"unknown case {case!r}")
    torch.cuda.synchronize()
    print(case, "ok")


if __name__ == "__main__":
    main(sys.argv[1])
