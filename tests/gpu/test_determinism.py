"""Repeat-run bit equality: the same inputs and launch give identical bits every time.

A race (a read before its producer finished, a lost update, an unordered
reduction) shows up as run-to-run differences, so each reducing kernel runs
many times on the same inputs and every result must equal the first one bit
for bit: the GEMM (single-CTA and CTA-pair tiles, fp32 accumulate), the
attention forward and deterministic backward, the RMSNorm backward (dw
partials + reduction), the embedding backward (sorted segment sums), the
cross-entropy and the grad-norm reduction.
"""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a GPU", allow_module_level=True)

from build_your_own_distributed_training_b200.ops import gemm  # noqa: E402
from build_your_own_distributed_training_b200.ops._ext import native  # noqa: E402

DEV = torch.device("cuda", 0)
BF = torch.bfloat16
RUNS = 100


def _same_every_time(fn, runs=RUNS):
    first = [t.clone() for t in fn()]
    for _ in range(runs - 1):
        for a, b in zip(first, fn()):
            assert torch.equal(a, b)
    assert native().device_error() == 0


def test_gemm_repeats_bitwise():
    g = torch.Generator(device=DEV).manual_seed(0)
    a = torch.randn(1000, 768, device=DEV, generator=g).to(BF)
    b = torch.randn(1536, 768, device=DEV, generator=g).to(BF)
    small = torch.randn(96, 768, device=DEV, generator=g).to(BF)

    def run():
        acc = torch.zeros(1536, 768, device=DEV)
        gemm.mm_tn_acc(gemm.mm_nt(a, b), a, acc)          # [1000,1536]^T x [1000,768]
        return [gemm.mm_nt(a, b), gemm.mm_nt(a, small), acc]
    _same_every_time(run)


def test_attention_repeats_bitwise():
    g = torch.Generator(device=DEV).manual_seed(1)
    b, s, nq, nkv, hd = 1, 512, 8, 2, 128
    qkv = torch.randn(b * s, (nq + 2 * nkv) * hd, device=DEV, generator=g).to(BF)
    do = torch.randn(b * s, nq * hd, device=DEV, generator=g).to(BF)
    sc = 1 / math.sqrt(hd)

    def run():
        o, lse = native().attn_fwd(qkv, b, s, nq, nkv, hd, sc)
        return [o, lse, native().attn_bwd(do, qkv, o, lse, b, s, nq, nkv, hd, sc)]
    _same_every_time(run, runs=30)


def test_reductions_repeat_bitwise():
    g = torch.Generator(device=DEV).manual_seed(2)
    x = torch.randn(4096, 1024, device=DEV, generator=g).to(BF)
    dy = torch.randn(4096, 1024, device=DEV, generator=g).to(BF)
    w = torch.randn(1024, device=DEV, generator=g).to(BF)
    tok = torch.randint(0, 500, (4096,), device=DEV, generator=g)
    logits = torch.randn(1024, 3000, device=DEV, generator=g)
    labels = torch.randint(0, 3000, (1024,), device=DEV, generator=g)
    big = torch.randn(1 << 22, device=DEV, generator=g)

    def run():
        _, rstd = native().rmsnorm_fwd(x, w, 1e-5)
        dw = torch.zeros(1024, device=DEV)
        dx = native().rmsnorm_bwd(dy, x, w, rstd, dw)
        emb = torch.zeros(500, 1024, device=DEV)
        native().embedding_bwd(tok, dy, emb)
        loss, dlog = native().cross_entropy_fwd(logits, labels, -100)
        return [dx, dw, emb, loss, dlog, native().sumsq(big)]
    _same_every_time(run)
