"""Small, self-contained launches of every native kernel, for ncu captures.

Each ``--case`` builds inputs of one 7B-layer shape (two 4096-token
sequences, 8192 rows; every case's inputs exceed the 126 MB L2 and hold a
few GB at most), launches the op once as warm-up, then ``--launches`` more
times, and checks the device error word.  It prints the CUDA-event time of
the timed launches.  Under ncu, skip the warm-up launches with ``-s``:

    python tests/performance/profile_kernels.py --case gemm_fwd
    ncu --set full --clock-control none -k regex:gemm_tcgen05 -s 1 -c 1 \\
        -o prof_gemm_fwd python tests/performance/profile_kernels.py --case gemm_fwd

The peer-memory kernels are emulated on one GPU: both "ranks'" symmetric
heaps are buffers on the local device, and the partner rank's flags are set
before launch, so the kernel runs its whole staging / flag / pull / sum path
with local HBM standing in for NVLink.
"""
import argparse
import math
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
import torch  # noqa: E402

from build_your_own_distributed_training_b200.ops import gemm  # noqa: E402
from build_your_own_distributed_training_b200.ops._ext import native  # noqa: E402
from build_your_own_distributed_training_b200.ops.rope import precompute_rope_cache  # noqa: E402

DEV = "cuda"
BF = torch.bfloat16
T = 8192          # tokens: 2 x 4096
D = 4096          # model width
FFN = 11008
V = 32000
HD = 128
HEADS = 32


def _bf(*shape):
    return torch.randn(*shape, device=DEV, dtype=BF)


def case_gemm_fwd():
    a, b = _bf(T, D), _bf(D, D)
    return lambda: gemm.mm_nt(a, b), 2 * T * D * D, 0


def case_gemm_residual():
    a, b, r = _bf(T, D), _bf(D, D), _bf(T, D)
    return lambda: gemm.mm_nt(a, b, residual=r), 2 * T * D * D, 0


def case_gemm_qkv_rope():
    a, b = _bf(T, D), _bf(3 * D, D)
    cos, sin = precompute_rope_cache(HD, 4096, 10000.0, device=DEV)
    return lambda: gemm.mm_nt_rope(a, b, cos, sin, 2 * D, HD, 4096), 2 * T * 3 * D * D, 0


def case_gemm_swiglu():
    a, b = _bf(T, D), _bf(2 * FFN, D)
    return lambda: gemm.mm_nt_swiglu(a, b, FFN), 2 * T * 2 * FFN * D, 0


def case_gemm_dgrad():
    dy, w = _bf(T, FFN), _bf(FFN, D)
    return lambda: gemm.mm_nn(dy, w), 2 * T * FFN * D, 0


def case_gemm_wgrad():
    dy, x = _bf(T, D), _bf(T, D)
    acc = torch.zeros(D, D, device=DEV)
    return lambda: gemm.mm_tn_acc(dy, x, acc), 2 * T * D * D, 0


def case_gemm_lm_head():
    h, w = _bf(T, D), _bf(V, D)
    return lambda: gemm.mm_nt(h, w, out_dtype=torch.float32), 2 * T * V * D, 0


def _emulated_heaps(world, nbytes):
    """``world`` heaps on this GPU; returns (heaps, bases)."""
    heaps = [torch.zeros(nbytes, device=DEV, dtype=torch.uint8) for _ in range(world)]
    return heaps, [int(h.data_ptr()) for h in heaps]


def case_gemm_peer_ar():
    # tp=2 row-parallel output projection: [T, D/2] x [D, D/2]^T, all-reduced
    a, b, r = _bf(T, D // 2), _bf(D, D // 2), _bf(T, D)
    out = torch.empty(T, D, device=DEV, dtype=BF)
    stage = T * D * 2
    flag_off = (stage + 255) // 256 * 256
    nflags = 2 * (T // 128) * (D // 128) * 4            # >= 2 ranks x tiles x quadrants
    heaps, bases = _emulated_heaps(2, flag_off + nflags * 4)
    heaps[1][:stage].view(BF).copy_(_bf(T * D))       # the partner's partial tile data
    epoch = [0]

    def run():
        epoch[0] += 1
        heaps[0][flag_off:].view(torch.int32).fill_(epoch[0])    # partner flags already published
        native().gemm_peer_ar(a, b, out, False, r, None, bases, 0, 0, flag_off, epoch[0], 1.0)
    return run, 2 * T * D * (D // 2), 0


def case_gemm_peer_rs():
    # tp=2 sequence-parallel output projection: [T, D/2] x [D, D/2]^T, reduce-scattered to rank 1's rows
    a, b = _bf(T, D // 2), _bf(D, D // 2)
    rows = T // 2
    r = _bf(rows, D)
    out = torch.empty(rows, D, device=DEV, dtype=BF)
    stage = T * D * 2
    flag_off = (stage + 255) // 256 * 256
    nflags = 2 * (T // 128 + 2) * (D // 128 + 2) * 4
    heaps, bases = _emulated_heaps(2, flag_off + nflags * 4)
    heaps[0][:stage].view(BF).copy_(_bf(T * D))       # rank 0's staged product
    epoch = [0]

    def run():
        epoch[0] += 1
        heaps[1][flag_off:].view(torch.int32).fill_(epoch[0])    # rank 0's flags already published
        native().gemm_peer_rs(a, b, out, False, r, bases, 1, 0, flag_off, epoch[0], 1.0, rows, rows)
    return run, 2 * T * D * (D // 2), 0


def case_gemm_peer_ar_two_shot():
    # tp=4 two-shot all-reduce epilogue, rank 0 with three emulated partners: [T, D/4] x [D, D/4]^T
    ranks = 4
    a, b, r = _bf(T, D // ranks), _bf(D, D // ranks), _bf(T, D)
    out = torch.empty(T, D, device=DEV, dtype=BF)
    stage = T * D * 2
    flag_off = (stage + 255) // 256 * 256
    nflags = 2 * (T // 128 + 2) * (D // 128 + 2) * 4
    heaps, bases = _emulated_heaps(ranks, flag_off + (ranks + 1) * nflags * 4)
    for p in range(1, ranks):
        heaps[p][:stage].view(BF).copy_(_bf(T * D))  # partials (read for rank 0's own units) / sums (copied)
    epoch = [0]

    def run():
        epoch[0] += 1
        heaps[0][flag_off:].view(torch.int32).fill_(epoch[0])    # partners' partial and done flags
        native().gemm_peer_ar(a, b, out, False, r, None, bases, 0, 0, flag_off, epoch[0], 1.0, two_shot=True)
    return run, 2 * T * D * (D // ranks), 0


def case_gemm_all_gather():
    # tp=2 sequence-parallel QKV input: rank 0 gathers [T, D] (its 4096 rows + the emulated
    # partner's staged rows) inside the GEMM, then [T, D] x [3D/2, D]^T
    ranks, R = 2, T // 2
    x_local = _bf(R, D)
    w = _bf(3 * D // 2, D)
    stage = R * D * 2
    staged_off = (stage + 255) // 256 * 256
    heaps, bases = _emulated_heaps(ranks, staged_off + 256)
    heaps[1][:stage].view(BF).copy_(_bf(R * D))
    xg = torch.empty(T, D, device=DEV, dtype=BF)
    out = torch.empty(T, 3 * D // 2, device=DEV, dtype=BF)
    epoch = [0]

    def run():
        epoch[0] += 1
        heaps[0][staged_off:staged_off + 4 * ranks].view(torch.int32).fill_(epoch[0])
        native().gemm_ag(xg, x_local, w, out, 0, None, None, None, 0, 0, bases, 0, 0, staged_off, epoch[0], 1.0)
    return run, 2 * T * D * (3 * D // 2), 0


def case_peer_all_gather():
    shard = 128 << 20
    heaps, bases = _emulated_heaps(2, shard)
    out = torch.empty(2 * shard, device=DEV, dtype=torch.uint8)
    return lambda: native().peer_all_gather(bases, 0, shard, out), 0, 3 * shard


def case_peer_reduce_scatter():
    n = 64 << 20                                      # fp32 elements per rank's full gradient
    heaps, bases = _emulated_heaps(2, n * 4)
    for h in heaps:
        h.view(torch.float32).normal_()
    out = torch.empty(n // 2, device=DEV)
    return lambda: native().peer_reduce_scatter(bases, 0, 0, 0.5, out), 0, 3 * (n // 2) * 4


def case_peer_all_reduce():
    n = T * D
    heaps, bases = _emulated_heaps(2, n * 2)
    out = torch.empty(n, device=DEV, dtype=BF)
    return lambda: native().peer_all_reduce_bf16(bases, 0, None, out), 0, 3 * n * 2


def case_peer_reduce_rows():
    n = T * D
    heaps, bases = _emulated_heaps(2, n * 2)
    out = torch.empty(T // 2, D, device=DEV, dtype=BF)
    return lambda: native().peer_reduce_rows_bf16(bases, 0, 0, D, out), 0, 3 * (n // 2) * 2


def _qkv():
    return _bf(4096, 3 * HEADS * HD)


def case_attn_fwd():
    qkv = _qkv()
    fl = 4 * HEADS * 4096 * 4096 * HD // 2
    return lambda: native().attn_fwd(qkv, 1, 4096, HEADS, HEADS, HD, 1 / math.sqrt(HD)), fl, 0


def case_attn_bwd():
    qkv = _qkv()
    o, lse = native().attn_fwd(qkv, 1, 4096, HEADS, HEADS, HD, 1 / math.sqrt(HD))
    do = torch.randn_like(o)
    fl = 5 * HEADS * 4096 * 4096 * HD
    return lambda: native().attn_bwd(do, qkv, o, lse, 1, 4096, HEADS, HEADS, HD, 1 / math.sqrt(HD)), fl, 0


def case_attn_legacy():
    # the mma.sync fallbacks serve sequence lengths that are a multiple of 64 but not of 128
    s = 4032
    qkv = _bf(s, 3 * HEADS * HD)
    o, lse = native().attn_fwd(qkv, 1, s, HEADS, HEADS, HD, 1 / math.sqrt(HD), legacy=True)
    do = torch.randn_like(o)

    def run():
        native().attn_fwd(qkv, 1, s, HEADS, HEADS, HD, 1 / math.sqrt(HD), legacy=True)
        native().attn_bwd(do, qkv, o, lse, 1, s, HEADS, HEADS, HD, 1 / math.sqrt(HD), legacy=True)
    return run, 7 * HEADS * s * s * HD, 0


def case_rmsnorm():
    x, w = _bf(T, D), torch.randn(D, device=DEV, dtype=BF)
    dy = _bf(T, D)
    acc = torch.zeros(D, device=DEV)

    def run():
        y, rstd = native().rmsnorm_fwd(x, w, 1e-5)
        native().rmsnorm_bwd(dy, x, w, rstd, acc)
    return run, 0, 5 * T * D * 2


def case_rope_bwd():
    d = _bf(T, 3 * D)
    cos, sin = precompute_rope_cache(HD, 4096, 10000.0, device=DEV)
    return lambda: native().rope_bwd(d, cos, sin, 2 * D, HD, 4096), 0, 2 * T * 2 * D * 2


def case_swiglu_bwd():
    da, gu = _bf(T, FFN), _bf(T, 2 * FFN)
    dgu = torch.empty_like(gu)
    return lambda: native().swiglu_bwd(da, gu, dgu), 0, T * FFN * 2 * 5


def case_embedding():
    tok = torch.randint(0, V, (T,), device=DEV)
    w = _bf(V, D)
    dout = _bf(T, D)
    acc = torch.zeros(V, D, device=DEV)

    def run():
        native().embedding_fwd(tok, w, BF)
        native().embedding_bwd(tok, dout, acc)
    return run, 0, 0


def case_cross_entropy():
    logits = torch.randn(T // 2, V, device=DEV)
    labels = torch.randint(0, V, (T // 2,), device=DEV)
    return lambda: native().cross_entropy_fwd(logits, labels, -100), 0, 2 * (T // 2) * V * 4


def case_ce_fused_fwd():
    # head GEMM with the log-sum-exp epilogue + row reduce + mean: 4096 tokens, V = 32000
    from build_your_own_distributed_training_b200.ops import loss as L
    h, w = _bf(T // 2, D), _bf(V, D)
    labels = torch.randint(0, V, (T // 2,), device=DEV)
    return lambda: L.fused_ce_forward(h, w, labels, 0, V), 2 * (T // 2) * V * D, 0


def case_ce_fused_bwd():
    # recomputed head GEMM writing bf16 logit-gradient chunks + dgrad + wgrad GEMMs
    from build_your_own_distributed_training_b200.ops import loss as L
    h, w = _bf(T // 2, D), _bf(V, D)
    labels = torch.randint(0, V, (T // 2,), device=DEV)
    _, lse, inv_n = L.fused_ce_forward(h, w, labels, 0, V)
    dloss = torch.ones((), device=DEV)
    mg = torch.zeros(V * D, device=DEV)
    return (lambda: L.fused_ce_backward(h, w, labels, lse, inv_n, dloss, 0, V, mg)), 3 * 2 * (T // 2) * V * D, 0


def case_sort_tokens():
    tok = torch.randint(0, V, (T,), device=DEV)
    dout = _bf(T, D)
    acc = torch.zeros(V, D, device=DEV)
    return lambda: native().embedding_bwd(tok, dout, acc), 0, 0


def case_adamw():
    n = 96 << 20
    p, g = torch.randn(n, device=DEV), torch.randn(n, device=DEV)
    m, v = torch.zeros(n, device=DEV), torch.zeros(n, device=DEV)
    out = torch.empty(n, device=DEV, dtype=BF)
    clip = torch.tensor([1.0, 1.0], device=DEV)
    return lambda: native().adamw(p, g, m, v, out, clip, 1e-4, 0.9, 0.95, 1e-8, 0.1, 1), 0, n * (16 + 12 + 2)


def case_sumsq():
    x = torch.randn(256 << 20, device=DEV)
    return lambda: native().sumsq(x), 0, x.numel() * 4


CASES = {k[5:]: v for k, v in globals().items() if k.startswith("case_")}


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--case", required=True, choices=sorted(CASES) + ["all"])
    p.add_argument("--launches", type=int, default=2)
    args = p.parse_args()
    names = sorted(CASES) if args.case == "all" else [args.case]
    for name in names:
        fn, flops, nbytes = CASES[name]()
        fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.launches):
            fn()
        e1.record()
        torch.cuda.synchronize()
        err = native().device_error()
        if err:
            raise SystemExit(f"{name}: device error word {err}")
        ms = e0.elapsed_time(e1) / args.launches
        extra = ""
        if flops:
            extra += f" {flops / ms / 1e9:.0f} TFLOP/s"
        if nbytes:
            extra += f" {nbytes / ms / 1e6:.0f} GB/s"
        print(f"{name}: {ms:.3f} ms{extra}", flush=True)


if __name__ == "__main__":
    main()
