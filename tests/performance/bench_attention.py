"""Flash-attention throughput: the tcgen05 forward/backward against the mma.sync kernels and
torch SDPA (the reference's attention kernel) on the same GPU.

    python tests/performance/bench_attention.py               # default kernels, mma.sync, SDPA
    python tests/performance/bench_attention.py --variants    # also every opt-in kernel variant

The kernel switches are read once per process, so ``--variants`` runs each variant in a child
process with its environment.  Times are CUDA events around 10 calls after 3 warm-ups; FLOPs
count the causal half (forward 4*b*h*s^2*hd/2, backward 2.5x the forward).
"""
import argparse
import math
import os
import subprocess
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
import torch  # noqa: E402
import torch.nn.functional as F  # noqa: E402

from build_your_own_distributed_training_b200.ops._ext import native  # noqa: E402

SHAPES = [(1, 4096, 32, 32, 128), (2, 4096, 16, 16, 128), (1, 8192, 4, 1, 128), (8, 2048, 6, 2, 64)]
VARIANTS = {
    "fwd_pp": {"DTB_ATTN_FWD_PP": "1"},          # two query tiles, P in shared memory
    "fwd_ws": {"DTB_ATTN_FWD_WS": "1"},          # two query tiles, P in tensor memory
    "bwd_early_s": {"DTB_ATTN_DKDV_EARLY_S": "1"},  # next S^T issued before this tile's dK
}


def tm(f, it=10):
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


def run(label: str, baselines: bool) -> None:
    for (b, s, nq, nkv, hd) in SHAPES:
        qkv = torch.randn(b * s, (nq + 2 * nkv) * hd, device="cuda", dtype=torch.bfloat16)
        scale = 1 / math.sqrt(hd)
        fl = 4 * b * nq * s * s * hd / 2
        t_f = tm(lambda: native().attn_fwd(qkv, b, s, nq, nkv, hd, scale))
        o, lse = native().attn_fwd(qkv, b, s, nq, nkv, hd, scale)
        do = torch.randn_like(o)
        t_b = tm(lambda: native().attn_bwd(do, qkv, o, lse, b, s, nq, nkv, hd, scale))
        line = f"[{label}] b{b} s{s} h{nq}/{nkv} hd{hd}: fwd {fl / t_f / 1e12:6.0f} TF/s | bwd {2.5 * fl / t_b / 1e12:6.0f}"
        if baselines:
            t_lg = tm(lambda: native().attn_fwd(qkv, b, s, nq, nkv, hd, scale, legacy=True))
            q = qkv[:, :nq * hd].view(b, s, nq, hd).transpose(1, 2).contiguous()
            k = qkv[:, nq * hd:(nq + nkv) * hd].view(b, s, nkv, hd).transpose(1, 2)
            v = qkv[:, (nq + nkv) * hd:].view(b, s, nkv, hd).transpose(1, 2)
            k = k.repeat_interleave(nq // nkv, 1).contiguous()
            v = v.repeat_interleave(nq // nkv, 1).contiguous()
            t_sd = tm(lambda: F.scaled_dot_product_attention(q, k, v, is_causal=True))
            qr, kr, vr = (x.detach().requires_grad_() for x in (q, k, v))
            out = F.scaled_dot_product_attention(qr, kr, vr, is_causal=True)
            go = torch.randn_like(out)
            t_sdb = tm(lambda: torch.autograd.grad(out, (qr, kr, vr), go, retain_graph=True))
            line += (f" | fwd mma.sync {fl / t_lg / 1e12:6.0f} | sdpa fwd {fl / t_sd / 1e12:6.0f}"
                     f" | sdpa bwd {2.5 * fl / t_sdb / 1e12:6.0f}")
        print(line, flush=True)
    assert native().device_error() == 0


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--variants", action="store_true", help="also time every opt-in kernel variant")
    ap.add_argument("--child", default=None, help=argparse.SUPPRESS)
    args = ap.parse_args()
    if args.child is not None:
        run(args.child, baselines=False)
        return
    run("default", baselines=True)
    if args.variants:
        for label, env in VARIANTS.items():
            r = subprocess.run([sys.executable, os.path.abspath(__file__), "--child", label],
                               env=dict(os.environ, **env), timeout=600)
            if r.returncode != 0:
                print(f"[{label}] failed with exit code {r.returncode}", flush=True)


if __name__ == "__main__":
    main()
