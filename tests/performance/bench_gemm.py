"""tcgen05 GEMM throughput vs torch.matmul (cuBLAS) on 7B layer shapes, all three layouts,
and the fused epilogues against the plain store on the same shape.

    python tests/performance/bench_gemm.py [--tokens 4096] [--tma-epi 0|1|2]

``--tma-epi`` sets the TMA-store epilogue level (0 row-per-thread stores, 1 the default,
2 also RoPE / SwiGLU).

CUDA events around 20 calls after 3 warm-ups; operands are 30-360 MB, so most of
each call's reads miss the 126 MB L2 (no separate flush).
"""
import argparse
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
import torch  # noqa: E402

from build_your_own_distributed_training_b200.ops import gemm  # noqa: E402
from build_your_own_distributed_training_b200.ops.rope import precompute_rope_cache  # noqa: E402

dev = "cuda"


def tm(f, it=20):
    for _ in range(3):
        f()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(it):
        f()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / it / 1e3


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=4096)
    ap.add_argument("--tma-epi", type=int, default=None)
    args = ap.parse_args()
    M = args.tokens
    if args.tma_epi is not None:
        from build_your_own_distributed_training_b200.ops._ext import native
        native().gemm_tma_epilogue(args.tma_epi)
    rows = []
    for (N, K) in [(12288, 4096), (4096, 4096), (22016, 4096), (4096, 11008), (32000, 4096)]:
        a = torch.randn(M, K, device=dev, dtype=torch.bfloat16)
        b = torch.randn(N, K, device=dev, dtype=torch.bfloat16)
        fl = 2 * M * N * K
        t_me = tm(lambda: gemm.mm_nt(a, b))
        t_cb = tm(lambda: a @ b.t())
        rows.append(("fwd nt", M, N, K, fl / t_me / 1e12, fl / t_cb / 1e12))
        if N == 12288:
            cos, sin = precompute_rope_cache(128, 4096, 10000.0)
            cos, sin = cos.to(dev).contiguous(), sin.to(dev).contiguous()
            t_r = tm(lambda: gemm.mm_nt_rope(a, b, cos, sin, 8192, 128, 4096))
            rows.append(("fwd nt+rope", M, N, K, fl / t_r / 1e12, fl / t_cb / 1e12))
        if N == 22016:
            t_s = tm(lambda: gemm.mm_nt_swiglu(a, b, N // 2))
            rows.append(("fwd nt+swiglu", M, N, K, fl / t_s / 1e12, fl / t_cb / 1e12))
        if N == 4096 and K == 4096:
            r = torch.randn(M, N, device=dev, dtype=torch.bfloat16)
            t_res = tm(lambda: gemm.mm_nt(a, b, residual=r))
            rows.append(("fwd nt+resid", M, N, K, fl / t_res / 1e12, fl / t_cb / 1e12))
        dy = torch.randn(M, N, device=dev, dtype=torch.bfloat16)
        t_me = tm(lambda: gemm.mm_nn(dy, b))
        t_cb = tm(lambda: dy @ b)
        rows.append(("dgrad nn", M, K, N, fl / t_me / 1e12, fl / t_cb / 1e12))
        acc = torch.zeros(N, K, device=dev)
        t_me = tm(lambda: gemm.mm_tn_acc(dy, a, acc))
        t_st = tm(lambda: gemm.mm_tn_acc(dy, a, acc, store=True))
        t_cb = tm(lambda: dy.t() @ a)
        rows.append(("wgrad tn+acc", N, K, M, fl / t_me / 1e12, fl / t_cb / 1e12))
        rows.append(("wgrad tn+store", N, K, M, fl / t_st / 1e12, fl / t_cb / 1e12))
        del a, b, dy, acc
        torch.cuda.empty_cache()
    for r in rows:
        print(f"{r[0]:15s} M={r[1]:6d} N={r[2]:6d} K={r[3]:6d}  mine {r[4]:7.1f} TF/s  cublas {r[5]:7.1f} TF/s  "
              f"ratio {r[4] / r[5]:.2f}", flush=True)


if __name__ == "__main__":
    main()
