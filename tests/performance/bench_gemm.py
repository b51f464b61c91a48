"""tcgen05 GEMM throughput vs torch.matmul (cuBLAS) on 7B layer shapes, all three layouts.

    python tests/performance/bench_gemm.py
"""
import os, sys
sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
import torch
from build_your_own_distributed_training_b200.ops import gemm
dev = "cuda"
def tm(f, it=20):
    for _ in range(3): f()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(it): f()
    e1.record(); torch.cuda.synchronize()
    return e0.elapsed_time(e1) / it / 1e3
M = 4096
rows = []
for (N, K) in [(12288, 4096), (4096, 4096), (22016, 4096), (4096, 11008), (32000, 4096)]:
    a = torch.randn(M, K, device=dev, dtype=torch.bfloat16); b = torch.randn(N, K, device=dev, dtype=torch.bfloat16)
    fl = 2 * M * N * K
    t_me = tm(lambda: gemm.mm_nt(a, b)); t_cb = tm(lambda: a @ b.t())
    rows.append(("fwd nt", M, N, K, fl / t_me / 1e12, fl / t_cb / 1e12))
    dy = torch.randn(M, N, device=dev, dtype=torch.bfloat16)
    t_me = tm(lambda: gemm.mm_nn(dy, b)); t_cb = tm(lambda: dy @ b)
    rows.append(("dgrad nn", M, K, N, fl / t_me / 1e12, fl / t_cb / 1e12))
    acc = torch.zeros(N, K, device=dev)
    t_me = tm(lambda: gemm.mm_tn_acc(dy, a, acc)); t_cb = tm(lambda: dy.t() @ a)
    rows.append(("wgrad tn+acc", N, K, M, fl / t_me / 1e12, fl / t_cb / 1e12))
for r in rows:
    print(f"{r[0]:14s} M={r[1]:6d} N={r[2]:6d} K={r[3]:6d}  mine {r[4]:7.1f} TF/s  cublas {r[5]:7.1f} TF/s  ratio {r[4]/r[5]:.2f}")
