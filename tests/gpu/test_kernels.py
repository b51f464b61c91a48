"""Numerics of every sm_100a kernel against a plain PyTorch fp32 restatement of the op."""

from __future__ import annotations

import math
import os

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover - collected on CPU boxes, skipped by marker
    pytest.skip("needs a GPU", allow_module_level=True)

# Kernel variants that are built but not yet the default (each behind its own switch) are
# checked only when DTB_TEST_OPT_IN=1, so that a variant still under development cannot fail
# a run of the default kernels.
opt_in = pytest.mark.skipif(os.environ.get("DTB_TEST_OPT_IN") != "1",
                            reason="opt-in kernel variant (DTB_TEST_OPT_IN=1 runs it)")

from build_your_own_distributed_training_b200.ops import gemm  # noqa: E402
from build_your_own_distributed_training_b200.ops._ext import native  # noqa: E402

DEV = torch.device("cuda", 0)
BF = torch.bfloat16


def _rel(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.float(), b.float()
    return float((a - b).norm() / b.norm().clamp_min(1e-12))


@pytest.fixture(autouse=True)
def _no_device_error():
    yield
    assert native().device_error() == 0


def _rand(*shape, scale=1.0):
    return (torch.randn(*shape, device=DEV) * scale).to(BF)


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (256, 512, 1024), (200, 384, 136), (4096, 4096, 4096),
                                   (1000, 96, 512), (64, 32000, 256)])
def test_gemm_nt(M, N, K):
    a, b = _rand(M, K), _rand(N, K)
    ref = a.float() @ b.float().t()
    out = gemm.mm_nt(a, b)
    assert out.dtype == BF
    assert _rel(out, ref) < 1e-2
    out32 = gemm.mm_nt(a, b, out_dtype=torch.float32)
    assert _rel(out32, ref) < 1e-5


@pytest.mark.parametrize("M,N,K", [(128, 128, 128), (512, 768, 256), (4096, 4096, 11008), (136, 200, 320)])
def test_gemm_nn(M, N, K):
    a, b = _rand(M, K), _rand(K, N)
    ref = a.float() @ b.float()
    assert _rel(gemm.mm_nn(a, b), ref) < 1e-2


@pytest.mark.parametrize("M,N,K", [(128, 128, 128), (768, 256, 512), (4096, 4096, 4096), (200, 136, 96)])
def test_gemm_tn_accumulate(M, N, K):
    a, b = _rand(K, M), _rand(K, N)
    acc = torch.randn(M, N, device=DEV)
    ref = acc + a.float().t() @ b.float()
    gemm.mm_tn_acc(a, b, acc)
    assert _rel(acc, ref) < 1e-5


@pytest.mark.parametrize("ks", [2, 3])
def test_gemm_wgrad_split_k_is_exact_order(ks):
    """The weight-gradient GEMM in K parts (DTB_GEMM_KSPLIT, read once per process: run in a
    child process) added in split order: both epilogues (store, accumulate) match the fp32
    oracle, with alpha, and repeat bit for bit."""
    import subprocess
    import sys
    code = ("import sys; sys.path.insert(0, %r)\n" % os.path.dirname(os.path.dirname(os.path.dirname(
        os.path.abspath(__file__)))) + "from tests.gpu.test_kernels import _split_k_case\n_split_k_case()\n")
    r = subprocess.run([sys.executable, "-c", code], env=dict(os.environ, DTB_GEMM_KSPLIT=str(ks)),
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "SPLITK_OK" in r.stdout, r.stdout[-2000:] + r.stderr[-2000:]


def _split_k_case():
    for (M, N, K) in [(4096, 4096, 4096), (1024, 4096, 8192), (4096, 3072, 2048)]:
        _split_k_shape(M, N, K)
    assert native().device_error() == 0
    print("SPLITK_OK")


def _split_k_shape(M, N, K):
    a, b = _rand(K, M), _rand(K, N)
    base = torch.randn(M, N, device=DEV)
    ref = a.float().t() @ b.float()
    st = torch.empty(M, N, device=DEV)
    gemm.mm_tn_acc(a, b, st, store=True)
    assert _rel(st, ref) < 1e-5
    acc = base.clone()
    gemm.mm_tn_acc(a, b, acc)
    assert _rel(acc, base + ref) < 1e-5
    alpha = torch.tensor([0.5], device=DEV)
    al = torch.empty(M, N, device=DEV)
    gemm.mm_tn_acc(a, b, al, alpha=alpha, store=True)
    assert _rel(al, 0.5 * ref) < 1e-5
    for _ in range(3):
        again = base.clone()
        gemm.mm_tn_acc(a, b, again)
        assert torch.equal(again, acc)


@pytest.mark.parametrize("M,N,K", [(200, 136, 96), (1000, 96, 512), (4096, 4096, 1024), (384, 4104, 256)])
def test_gemm_tma_epilogues_match_row_path(M, N, K):
    """Store (bf16, fp32), TMA reduce-add accumulate and residual epilogues through TMA
    boxes give the same bits as the row-per-thread epilogues, and match the fp32 oracle;
    partial boxes at the right and bottom edges are clipped by the tensor map."""
    a, b, r = _rand(M, K), _rand(N, K), _rand(M, N)
    at, bt = _rand(K, M), _rand(K, N)
    alpha = torch.tensor([0.375], device=DEV)
    base = torch.randn(M, N, device=DEV)

    def run():
        out = {}
        out["bf16"] = gemm.mm_nt(a, b)
        out["f32"] = gemm.mm_nt(a, b, out_dtype=torch.float32)
        res = torch.empty(M, N, device=DEV, dtype=BF)
        native().gemm(a, b, res, False, False, gemm.EPI_RESIDUAL, r, alpha, None, None, None, 0, 0)
        out["res"] = res
        acc = base.clone()
        gemm.mm_tn_acc(at, bt, acc, alpha=alpha)
        out["acc"] = acc
        st = torch.empty(M, N, device=DEV)
        gemm.mm_tn_acc(at, bt, st, store=True)
        out["st"] = st
        return out

    prev = native().gemm_tma_epilogue(1)
    try:
        tma = run()
        native().gemm_tma_epilogue(0)
        row = run()
    finally:
        native().gemm_tma_epilogue(prev)
    for k in tma:
        assert torch.equal(tma[k], row[k]), k
    ref = a.float() @ b.float().t()
    reft = at.float().t() @ bt.float()
    assert _rel(tma["bf16"], ref) < 1e-2
    assert _rel(tma["f32"], ref) < 1e-5
    assert _rel(tma["res"], 0.375 * ref + r.float()) < 1e-2
    assert _rel(tma["acc"], base + 0.375 * reft) < 1e-5
    assert _rel(tma["st"], reft) < 1e-5


@opt_in
@pytest.mark.parametrize("M,hd,seq", [(512, 128, 256), (300, 64, 300)])
def test_gemm_tma_rope_swiglu_match_row_path(M, hd, seq):
    """The RoPE and SwiGLU epilogues through TMA boxes (epilogue level 2, not yet the
    default) give the row-per-thread bits.  Runs in a child process, so that a failure
    of the new path cannot take this process's CUDA context with it."""
    import subprocess
    import sys
    code = ("import sys; sys.path.insert(0, %r)\n" % os.path.dirname(os.path.dirname(os.path.dirname(
        os.path.abspath(__file__)))) + "from tests.gpu.test_kernels import _tma_rope_swiglu_case\n"
        "_tma_rope_swiglu_case(%d, %d, %d)\n" % (M, hd, seq))
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "TMA_ROPE_SWIGLU_OK" in r.stdout, r.stdout[-2000:] + r.stderr[-2000:]


def _tma_rope_swiglu_case(M, hd, seq):
    from build_your_own_distributed_training_b200.ops.rope import precompute_rope_cache
    K, heads, ffn = 256, 4, 384
    a = _rand(M, K)
    wqkv = _rand(3 * heads * hd, K, scale=0.1)
    wgu = _rand(2 * ffn, K, scale=0.1)
    cos, sin = precompute_rope_cache(hd, seq, 10000.0, device=DEV)

    def run():
        q = gemm.mm_nt_rope(a, wqkv, cos, sin, 2 * heads * hd, hd, seq)
        act, gu = gemm.mm_nt_swiglu(a, wgu, ffn)
        return q, act, gu

    native().gemm_tma_epilogue(2)
    tma = run()
    native().gemm_tma_epilogue(0)
    row = run()
    for name, x, y in zip(("rope", "act", "gu"), tma, row):
        assert torch.equal(x, y), name
    g, u = (a.float() @ wgu.float().t()).split(ffn, dim=1)
    assert _rel(tma[2], torch.cat([g, u], 1)) < 1e-2
    gr, ur = tma[2].float().split(ffn, dim=1)
    assert _rel(tma[1], torch.nn.functional.silu(gr) * ur) < 1e-2
    assert native().device_error() == 0
    print("TMA_ROPE_SWIGLU_OK")


def test_tmem_a_operand_layout():
    """tcgen05 MMA reading A from tensor memory in the softmax threads' layout (row = lane,
    bf16 pairs per 32-bit column) equals the fp32 product."""
    a, b = _rand(128, 128), _rand(128, 128)
    d = native().tmem_a_operand_check(a, b)
    assert _rel(d, a.float() @ b.float().t()) < 1e-5


def test_gemm_alpha_and_residual():
    a, b, r = _rand(256, 512), _rand(384, 512), _rand(256, 384)
    alpha = torch.tensor([0.25], device=DEV)
    ref = 0.25 * (a.float() @ b.float().t()) + r.float()
    # alpha applies before the residual add
    out = torch.empty(256, 384, device=DEV, dtype=BF)
    native().gemm(a, b, out, False, False, gemm.EPI_RESIDUAL, r, alpha, None, None, None, 0, 0)
    assert _rel(out, ref) < 1e-2


@pytest.mark.parametrize("hd,nq,nkv", [(128, 4, 4), (64, 8, 2)])
def test_gemm_rope_epilogue(hd, nq, nkv):
    from build_your_own_distributed_training_b200.ops.rope import precompute_rope_cache, rope_forward
    seqlen, b, d = 256, 2, 512
    x, w = _rand(b * seqlen, d), _rand((nq + 2 * nkv) * hd, d, scale=0.05)
    cos, sin = precompute_rope_cache(hd, 512, 10000.0, DEV)
    rope_cols = (nq + nkv) * hd
    out = gemm.mm_nt_rope(x, w, cos, sin, rope_cols, hd, seqlen)
    ref = x.float() @ w.float().t()
    rope_forward(ref, cos, sin, rope_cols, hd, seqlen)
    assert _rel(out, ref) < 1e-2


def test_gemm_swiglu_epilogue():
    M, K, Fh = 512, 256, 384
    x, w = _rand(M, K), _rand(2 * Fh, K, scale=0.1)
    act, gu = gemm.mm_nt_swiglu(x, w, Fh)
    ref_gu = x.float() @ w.float().t()
    ref = F.silu(ref_gu[:, :Fh]) * ref_gu[:, Fh:]
    assert _rel(gu, ref_gu) < 1e-2
    assert _rel(act, ref) < 2e-2


@pytest.mark.parametrize("M,N,K", [(1024, 1024, 512), (200, 384, 256), (4096, 4096, 2048)])
def test_gemm_peer_allreduce_emulated_partner(M, N, K):
    """The fused GEMM + all-reduce on one GPU, the partner rank emulated by memory.

    Two "ranks'" symmetric heaps are local buffers; the partner's staged
    partial tile holds known data and its flags are set before the launch, so
    rank 0's kernel runs its whole stage / publish / wait / pull / sum path.
    """
    a, b, r = _rand(M, K), _rand(N, K), _rand(M, N)
    partner = _rand(M, N)
    stage = M * N * 2
    flag_off = (stage + 255) // 256 * 256
    nflags = 2 * (M // 128 + 2) * (N // 128 + 2) * 4
    heaps = [torch.zeros(flag_off + nflags * 4, device=DEV, dtype=torch.uint8) for _ in range(2)]
    heaps[1][:stage].view(BF).copy_(partner.reshape(-1))
    heaps[0][flag_off:].view(torch.int32).fill_(7)
    out = torch.empty(M, N, device=DEV, dtype=BF)
    native().gemm_peer_ar(a, b, out, False, r, None, [h.data_ptr() for h in heaps], 0, 0, flag_off, 7, 1.0)
    mine = (a.float() @ b.float().t()).to(BF).float()
    ref = mine + partner.float() + r.float()
    assert _rel(out, ref) < 1e-2
    # rank 0 published its own tile to the partner's flag array
    assert int((heaps[1][flag_off:].view(torch.int32) == 7).sum()) > 0


def _two_shot_owner_map(M: int, N: int, ranks: int) -> torch.Tensor:
    """Owner rank of every (32-row group, output column) under the two-shot schedule:
    the (tile, quadrant) unit f belongs to rank f % ranks (csrc/gemm.cu two_shot_owner)."""
    BN = 256 if N > 128 else 128
    pair = BN == 256 and M > 128 and os.environ.get("DTB_GEMM_PAIR", "1") != "0"
    tile_m = 256 if pair else 128
    mblocks, nblocks = -(-M // tile_m), -(-N // BN)
    own = torch.empty(-(-M // 32) + 8, N, dtype=torch.int64)
    for tile in range(mblocks * nblocks):
        per_group = 16 * nblocks
        g = tile // per_group
        gm = min(16, mblocks - g * 16)
        r = tile - g * per_group
        mb, nb = g * 16 + r % gm, r // gm
        for cta in range(2 if pair else 1):
            ftile = 2 * tile + cta if pair else tile
            slab = 2 * mb + cta if pair else mb
            for q in range(4):
                own[slab * 4 + q, nb * BN:(nb + 1) * BN] = (ftile * 4 + q) % ranks
    return own[:-(-M // 32)].repeat_interleave(32, dim=0)[:M]


@pytest.mark.parametrize("M,N,K", [(1024, 1024, 512), (200, 384, 256), (4096, 4096, 2048)])
def test_gemm_peer_allreduce_two_shot_emulated_partner(M, N, K):
    """Two-shot fused all-reduce, rank 0 of 2 with the partner emulated by memory: rank 0 sums the
    units it owns (and writes the sum back to its staging) and copies the partner's units from the
    partner's staging, where the emulated partner has already left its sum."""
    a, b, r = _rand(M, K), _rand(N, K), _rand(M, N)
    partner = _rand(M, N)
    stage = M * N * 2
    flag_off = (stage + 255) // 256 * 256
    nflags = 2 * (M // 128 + 2) * (N // 128 + 2) * 4
    heaps = [torch.zeros(flag_off + 3 * nflags * 4, device=DEV, dtype=torch.uint8) for _ in range(2)]
    heaps[1][:stage].view(BF).copy_(partner.reshape(-1))
    heaps[0][flag_off:].view(torch.int32).fill_(9)  # partner's partial flags and done flags
    out = torch.empty(M, N, device=DEV, dtype=BF)
    native().gemm_peer_ar(a, b, out, False, r, None, [h.data_ptr() for h in heaps], 0, 0, flag_off, 9, 1.0,
                          two_shot=True)
    mine = (a.float() @ b.float().t()).to(BF).float()
    own = _two_shot_owner_map(M, N, 2).to(DEV)
    ref = torch.where(own == 0, mine + partner.float() + r.float(), partner.float())
    assert _rel(out, ref) < 1e-2
    assert (own == 0).any() and (own == 1).any()
    staged0 = heaps[0][:stage].view(BF).view(M, N)
    assert torch.equal(staged0[own == 0], out[own == 0])  # the owner's sum, for the partner to copy


@pytest.mark.parametrize("ranks,R,N,K,epi", [(2, 512, 768, 512, "store"), (4, 256, 512, 1024, "store"),
                                              (2, 1024, 4096, 4096, "store"), (2, 512, 1024, 512, "swiglu"),
                                              (2, 256, 768, 256, "rope")])
def test_gemm_all_gather_emulated_peers(ranks, R, N, K, epi):
    """The all-gather fused in front of the GEMM, rank 0 of `ranks` with the peers emulated by
    memory: their rows sit staged in their heaps and their staged flags are raised before the
    launch, so the copier warps pull them while the tiles of rank 0's own rows start."""
    M = ranks * R
    x = _rand(M, K)
    w = _rand(N, K, scale=0.5)
    stage = R * K * 2
    staged_off = (stage + 255) // 256 * 256
    heaps = [torch.zeros(staged_off + 256, device=DEV, dtype=torch.uint8) for _ in range(ranks)]
    for p in range(1, ranks):
        heaps[p][:stage].view(BF).copy_(x[p * R:(p + 1) * R].reshape(-1))
    heaps[0][staged_off:staged_off + 4 * ranks].view(torch.int32).fill_(3)
    xg = torch.empty(M, K, device=DEV, dtype=BF)
    bases = [h.data_ptr() for h in heaps]
    if epi == "store":
        out = torch.empty(M, N, device=DEV, dtype=BF)
        native().gemm_ag(xg, x[:R].contiguous(), w, out, 0, None, None, None, 0, 0, bases, 0, 0, staged_off, 3, 2.0)
        ref = x.float() @ w.float().t()
    elif epi == "swiglu":
        F2 = N // 2
        out = torch.empty(M, F2, device=DEV, dtype=BF)
        gu = torch.empty(M, N, device=DEV, dtype=BF)
        native().gemm_ag(xg, x[:R].contiguous(), w, out, 5, None, None, gu, F2, 0, bases, 0, 0, staged_off, 3, 2.0)
        y = x.float() @ w.float().t()
        ref = torch.nn.functional.silu(y[:, :F2]) * y[:, F2:]
    else:
        from build_your_own_distributed_training_b200.ops.rope import precompute_rope_cache
        hd, seq = 128, 256
        cos, sin = precompute_rope_cache(hd, seq, 10000.0, device=DEV)
        out = torch.empty(M, N, device=DEV, dtype=BF)
        native().gemm_ag(xg, x[:R].contiguous(), w, out, 4, cos, sin, None, 2 * hd * 2, hd * 65536 + seq, bases, 0,
                         0, staged_off, 3, 2.0)
        ref = gemm.mm_nt_rope(x, w, cos, sin, 2 * hd * 2, hd, seq).float()
    assert torch.equal(xg, x)  # the gathered rows are the GEMM's saved input for the weight gradient
    assert _rel(out, ref) < 2e-2


@pytest.mark.parametrize("M,N,K", [(1024, 768, 512), (4096, 4096, 2048)])
def test_gemm_peer_reduce_scatter_emulated_partner(M, N, K):
    """The fused GEMM + reduce-scatter of rows on one GPU, the partner emulated by memory:
    rank 1 of 2 sums only its row block (the second half) and adds the scattered residual."""
    a, b = _rand(M, K), _rand(N, K)
    rows = M // 2
    r = _rand(rows, N)
    partner = _rand(M, N)
    stage = M * N * 2
    flag_off = (stage + 255) // 256 * 256
    nflags = 2 * (M // 128 + 2) * (N // 128 + 2) * 4
    heaps = [torch.zeros(flag_off + nflags * 4, device=DEV, dtype=torch.uint8) for _ in range(2)]
    heaps[0][:stage].view(BF).copy_(partner.reshape(-1))   # rank 0's staged product
    heaps[1][flag_off:].view(torch.int32).fill_(5)          # rank 0's flags, as seen by rank 1
    out = torch.empty(rows, N, device=DEV, dtype=BF)
    native().gemm_peer_rs(a, b, out, False, r, [h.data_ptr() for h in heaps], 1, 0, flag_off, 5, 1.0, rows, rows)
    mine = (a.float() @ b.float().t()).to(BF).float()
    ref = partner.float()[rows:] + mine[rows:] + r.float()
    assert _rel(out, ref) < 1e-2


@pytest.mark.parametrize("M,D,wdt", [(1000, 4096, BF), (1001, 2048, torch.float32), (333, 1536, BF),
                                     (64, 8192, BF)])
def test_rmsnorm_fwd_bwd(M, D, wdt):
    """Register-resident kernels for the usual widths, the general kernels otherwise (D = 1536)."""
    from build_your_own_distributed_training_b200.ops.norm import rms_norm
    x = _rand(M, D).requires_grad_()
    w = (1 + 0.1 * torch.randn(D, device=DEV)).to(wdt).requires_grad_()
    y = rms_norm(x, w, 1e-5)
    xr = x.detach().float().requires_grad_()
    wr = w.detach().float().requires_grad_()
    yr = xr * torch.rsqrt(xr.pow(2).mean(-1, keepdim=True) + 1e-5) * wr
    assert _rel(y, yr) < 1e-2
    g = torch.randn_like(yr)
    y.backward(g.to(BF))
    yr.backward(g)
    assert _rel(x.grad, xr.grad) < 2e-2
    assert _rel(w.grad, wr.grad) < 2e-2


def test_rmsnorm_backward_is_deterministic():
    from build_your_own_distributed_training_b200.ops.norm import _RMSNormFn
    x = _rand(4096, 4096)
    w = torch.ones(4096, device=DEV, dtype=BF)
    dy = _rand(4096, 4096)
    outs = []
    for _ in range(3):
        acc = torch.zeros(4096, device=DEV)
        _, rstd = native().rmsnorm_fwd(x, w, 1e-5)
        dx = native().rmsnorm_bwd(dy, x, w, rstd, acc)
        outs.append((dx, acc))
    for dx, acc in outs[1:]:
        assert torch.equal(dx, outs[0][0]) and torch.equal(acc, outs[0][1])
    del _RMSNormFn


@pytest.mark.parametrize("pad", [0, 4])
def test_rope_bwd_is_transpose(pad):
    """pad=0: 16-byte vector kernel; pad=4 (rows not 16-byte aligned): the scalar kernel."""
    from build_your_own_distributed_training_b200.ops.rope import precompute_rope_cache, rope_backward_, rope_forward
    hd, seqlen = 128, 128
    cos, sin = precompute_rope_cache(hd, 256, 10000.0, DEV)
    base = _rand(2 * seqlen, 6 * hd + pad)
    d = base[:, :6 * hd]
    ref = d.float().cpu().clone()
    rope_backward_(ref, cos.cpu(), sin.cpu(), 4 * hd, hd, seqlen)
    out = base.clone()[:, :6 * hd]  # keeps the padded row stride
    rope_backward_(out, cos, sin, 4 * hd, hd, seqlen)
    assert _rel(out.cpu(), ref) < 1e-2
    # forward then backward is the identity (rotation is orthogonal)
    y = d.float().cpu()
    rope_forward(y, cos.cpu(), sin.cpu(), 4 * hd, hd, seqlen)
    rope_backward_(y, cos.cpu(), sin.cpu(), 4 * hd, hd, seqlen)
    assert _rel(y, d.float().cpu()) < 1e-5


@pytest.mark.parametrize("Fh", [256, 100])
def test_swiglu_bwd(Fh):
    """Fh % 8 == 0: 16-byte vector kernel; Fh = 100: the two-element kernel."""
    from build_your_own_distributed_training_b200.ops.linear import swiglu_backward
    M = 300
    gu, da = _rand(M, 2 * Fh), _rand(M, Fh)
    out = swiglu_backward(da, gu, Fh)
    ref = swiglu_backward(da.cpu().float(), gu.cpu().float(), Fh)
    assert _rel(out.cpu(), ref) < 1e-2


def test_embedding_fwd_bwd_deterministic():
    V, D, M = 1000, 256, 4096
    w = _rand(V, D)
    tok = torch.randint(0, V, (M,), device=DEV)
    out = native().embedding_fwd(tok, w, BF)
    assert torch.equal(out, w[tok])
    dout = _rand(M, D)
    accs = []
    for _ in range(2):
        acc = torch.zeros(V, D, device=DEV)
        native().embedding_bwd(tok, dout, acc)
        accs.append(acc)
    ref = torch.zeros(V, D, device=DEV).index_add_(0, tok, dout.float())
    assert _rel(accs[0], ref) < 1e-5
    assert torch.equal(accs[0], accs[1])


@pytest.mark.parametrize("M,V", [(512, 32000), (100, 1000)])
def test_cross_entropy(M, V):
    logits = torch.randn(M, V, device=DEV) * 3
    labels = torch.randint(0, V, (M,), device=DEV)
    labels[::7] = -100
    loss, dlog = native().cross_entropy_fwd(logits, labels, -100)
    lr = logits.clone().requires_grad_()
    ref = F.cross_entropy(lr, labels, ignore_index=-100)
    ref.backward()
    assert abs(float(loss) - float(ref)) < 1e-4 * max(1.0, float(ref))
    assert _rel(dlog, lr.grad) < 1e-2


@pytest.mark.parametrize("M,V,d,chunk", [(512, 32000, 256, 8192), (384, 128256, 128, 8192), (200, 1000, 64, 256),
                                         (256, 4096, 128, 100000)])
def test_fused_head_cross_entropy(M, V, d, chunk):
    """Head GEMM + CE without logits vs the fp32 oracle F.cross_entropy(h W^T)."""
    from build_your_own_distributed_training_b200.ops import loss as L
    torch.manual_seed(0)
    h = _rand(M, d)
    w = _rand(V, d, scale=0.5)
    labels = torch.randint(0, V, (M,), device=DEV)
    labels[::7] = -100
    labels[0] = V - 1  # last column of the last chunk / block
    loss, lse, inv_n = L.fused_ce_forward(h, w, labels, 0, V)
    hf, wf = h.float().requires_grad_(), w.float().requires_grad_()
    logits = hf @ wf.t()
    ref = F.cross_entropy(logits, labels, ignore_index=-100)
    ref.backward()
    assert abs(float(loss) - float(ref)) < 2e-4 * max(1.0, float(ref))
    assert _rel(lse, torch.logsumexp(logits.detach(), dim=1)) < 1e-5
    assert abs(float(inv_n) - 1.0 / int((labels != -100).sum())) < 1e-9
    dloss = torch.full((), 0.75, device=DEV)
    dh, dw = L.fused_ce_backward(h, w, labels, lse, inv_n, dloss, 0, V, None, chunk=chunk)
    assert _rel(dh, 0.75 * hf.grad) < 2e-2
    assert _rel(dw, 0.75 * wf.grad) < 2e-2
    # into a main_grad slice: overwritten while fresh, accumulated afterwards
    mg = torch.full((V * d,), 3.0, device=DEV)
    from build_your_own_distributed_training_b200.ops import grad_state
    fs = grad_state.FreshSet(mg)
    fs.mark([(0, V * d)])
    grad_state.tag(mg, fs, 0)
    _, none = L.fused_ce_backward(h, w, labels, lse, inv_n, dloss, 0, V, mg, chunk=chunk)
    assert none is None and _rel(mg.view(V, d), 0.75 * wf.grad) < 2e-2
    L.fused_ce_backward(h, w, labels, lse, inv_n, dloss, 0, V, mg, chunk=chunk)
    assert _rel(mg.view(V, d), 1.5 * wf.grad) < 2e-2


def test_fused_head_cross_entropy_vocab_split_matches_whole():
    """Two vocabulary halves combined through the row-record exchange equal the whole-vocabulary loss."""
    from build_your_own_distributed_training_b200.ops import loss as L
    torch.manual_seed(1)
    M, V, d = 300, 2048, 128
    h, w = _rand(M, d), _rand(V, d, scale=0.5)
    labels = torch.randint(0, V, (M,), device=DEV)
    labels[::5] = -100
    loss, lse, inv_n = L.fused_ce_forward(h, w, labels, 0, V)

    class TwoHalves:  # both "ranks" on one GPU: records of half 0 and half 1 side by side
        def __init__(self):
            self.buf = torch.zeros(2, M * 4, device=DEV)
            self.r = 0

        def exchange_rows(self, rows, nb):
            return 0, self.buf[self.r]

        def exchange_publish(self, off, rows):
            return [self.buf[0].data_ptr(), self.buf[1].data_ptr()], 0

    ex = TwoHalves()
    ex.r = 1
    L.fused_ce_forward(h, w[V // 2:], labels, V // 2, V, ex)  # fills half 1's records
    ex.r = 0
    loss0, lse0, inv0 = L.fused_ce_forward(h, w[:V // 2], labels, 0, V, ex)
    assert abs(float(loss0) - float(loss)) < 1e-5 * max(1.0, float(loss))
    assert _rel(lse0, lse) < 1e-6 and float(inv0) == float(inv_n)
    dloss = torch.ones((), device=DEV)
    dh, dw = L.fused_ce_backward(h, w, labels, lse, inv_n, dloss, 0, V, None)
    dh0, dw0 = L.fused_ce_backward(h, w[:V // 2], labels, lse0, inv0, dloss, 0, V, None)
    dh1, dw1 = L.fused_ce_backward(h, w[V // 2:], labels, lse0, inv0, dloss, V // 2, V, None)
    assert _rel(dh0.float() + dh1.float(), dh) < 1e-2
    assert _rel(torch.cat([dw0, dw1]), dw) < 1e-3


def test_adamw_matches_torch():
    n = 100_003
    p = torch.randn(n, device=DEV)
    g = torch.randn(n, device=DEV)
    m, v = torch.zeros(n, device=DEV), torch.zeros(n, device=DEV)
    out = torch.empty(n, device=DEV, dtype=BF)
    ref = p.clone().requires_grad_()
    opt = torch.optim.AdamW([ref], lr=1e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)
    clip = torch.tensor([0.5, 1.0], device=DEV)
    for step in range(1, 4):
        ref.grad = g * 0.5
        opt.step()
        native().adamw(p, g, m, v, out, clip, 1e-3, 0.9, 0.95, 1e-8, 0.1, step)
    assert _rel(p, ref.detach()) < 1e-6
    assert torch.equal(out, p.to(BF))
    # non-finite flag skips the update
    before = p.clone()
    native().adamw(p, g, m, v, out, torch.tensor([0.0, 0.0], device=DEV), 1e-3, 0.9, 0.95, 1e-8, 0.1, 4)
    assert torch.equal(p, before)


def test_sumsq():
    x = torch.randn(10_000_019, device=DEV)
    s = native().sumsq(x)
    assert abs(float(s) - float(x.double().pow(2).sum())) / float(x.double().pow(2).sum()) < 1e-5
    assert torch.equal(s, native().sumsq(x))


def _attn_ref(qkv, b, s, nq, nkv, hd):
    from build_your_own_distributed_training_b200.ops.attention import attention_reference
    return attention_reference(qkv.float(), b, s, nq, nkv, hd)


@pytest.mark.parametrize("b,s,nq,nkv,hd", [(2, 128, 4, 4, 128), (1, 256, 8, 2, 64), (2, 192, 4, 1, 128),
                                           (1, 1024, 2, 2, 128),
                                           # head sizes and ragged lengths of the mma.sync kernels
                                           (4, 64, 4, 2, 16), (2, 96, 4, 2, 16), (3, 200, 4, 4, 32),
                                           (2, 77, 2, 1, 64), (1, 130, 4, 2, 128), (2, 1, 2, 2, 32)])
def test_attention_fwd_bwd(b, s, nq, nkv, hd):
    from build_your_own_distributed_training_b200.ops.attention import causal_attention
    qkv = _rand(b * s, (nq + 2 * nkv) * hd).requires_grad_()
    o = causal_attention(qkv, b, s, nq, nkv, hd)
    ref_in = qkv.detach().float().requires_grad_()
    ref = _attn_ref(ref_in, b, s, nq, nkv, hd)
    assert _rel(o, ref) < 2e-2
    do = torch.randn_like(ref)
    o.backward(do.to(BF))
    ref.backward(do)
    assert _rel(qkv.grad, ref_in.grad) < 3e-2
    # bit-reproducible backward
    g1 = qkv.grad.clone()
    qkv.grad = None
    causal_attention(qkv, b, s, nq, nkv, hd).backward(do.to(BF))
    assert torch.equal(qkv.grad, g1)


def test_attention_lse_scale():
    b, s, nq, nkv, hd = 1, 128, 2, 2, 64
    qkv = _rand(b * s, (nq + 2 * nkv) * hd)
    o, lse = native().attn_fwd(qkv, b, s, nq, nkv, hd, 1 / math.sqrt(hd))
    q = qkv.float()[:, :nq * hd].view(s, nq, hd).transpose(0, 1)
    k = qkv.float()[:, nq * hd:(nq + nkv) * hd].view(s, nkv, hd).transpose(0, 1)
    sc = q @ k.transpose(1, 2) / math.sqrt(hd)
    sc = sc.masked_fill(torch.triu(torch.ones(s, s, device=DEV, dtype=torch.bool), 1), float("-inf"))
    assert _rel(lse[0], torch.logsumexp(sc, -1)) < 1e-4


@pytest.mark.parametrize("b,s,nq,nkv,hd", [(1, 128, 2, 2, 128), (2, 256, 4, 2, 128), (1, 512, 8, 2, 64),
                                           (1, 1024, 4, 4, 128), (2, 384, 2, 1, 64)])
def test_attention_tcgen05_forward(b, s, nq, nkv, hd):
    qkv = _rand(b * s, (nq + 2 * nkv) * hd)
    scale = 1 / math.sqrt(hd)
    o, lse = native().attn_fwd(qkv, b, s, nq, nkv, hd, scale)
    o_legacy, lse_legacy = native().attn_fwd(qkv, b, s, nq, nkv, hd, scale, legacy=True)
    ref = _attn_ref(qkv, b, s, nq, nkv, hd)
    assert _rel(o, ref) < 2e-2
    assert _rel(o, o_legacy) < 2e-2
    assert _rel(lse, lse_legacy) < 1e-4


@pytest.mark.parametrize("b,s,nq,nkv,hd", [(1, 128, 2, 2, 128), (2, 256, 4, 2, 128), (1, 512, 8, 2, 64),
                                           (1, 1024, 4, 4, 128)])
def test_attention_tcgen05_backward(b, s, nq, nkv, hd):
    qkv = _rand(b * s, (nq + 2 * nkv) * hd)
    scale = 1 / math.sqrt(hd)
    o, lse = native().attn_fwd(qkv, b, s, nq, nkv, hd, scale)
    do = _rand(b * s, nq * hd)
    d_tc = native().attn_bwd(do, qkv, o, lse, b, s, nq, nkv, hd, scale)
    d_legacy = native().attn_bwd(do, qkv, o, lse, b, s, nq, nkv, hd, scale, legacy=True)
    ref_in = qkv.detach().float().requires_grad_()
    _attn_ref(ref_in, b, s, nq, nkv, hd).backward(do.float())
    assert _rel(d_tc, ref_in.grad) < 3e-2
    assert _rel(d_tc, d_legacy) < 2e-2
    assert torch.equal(d_tc, native().attn_bwd(do, qkv, o, lse, b, s, nq, nkv, hd, scale))


@opt_in
def test_attention_forward_two_tiles_p_in_tmem():
    """The forward with two query tiles per CTA and P kept in tensor memory
    (DTB_ATTN_FWD_WS=1, read once per process: run in a child process) matches the fp32
    oracle and the default forward's log-sum-exp."""
    import subprocess
    import sys
    code = ("import sys; sys.path.insert(0, %r)\n" % os.path.dirname(os.path.dirname(os.path.dirname(
        os.path.abspath(__file__)))) + "from tests.gpu.test_kernels import _attn_fwd_ws_case\n_attn_fwd_ws_case()\n")
    r = subprocess.run([sys.executable, "-c", code], env=dict(os.environ, DTB_ATTN_FWD_WS="1"),
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "ATTN_FWD_WS_OK" in r.stdout, r.stdout[-2000:] + r.stderr[-2000:]


def _attn_fwd_ws_case():
    for (b, s, nq, nkv, hd) in [(1, 256, 2, 2, 128), (2, 512, 4, 2, 128), (1, 1024, 8, 2, 64), (1, 768, 4, 4, 128)]:
        qkv = _rand(b * s, (nq + 2 * nkv) * hd)
        scale = 1 / math.sqrt(hd)
        o, lse = native().attn_fwd(qkv, b, s, nq, nkv, hd, scale)
        o_legacy, lse_legacy = native().attn_fwd(qkv, b, s, nq, nkv, hd, scale, legacy=True)
        assert _rel(o, _attn_ref(qkv, b, s, nq, nkv, hd)) < 2e-2, (b, s, nq, nkv, hd)
        assert _rel(o, o_legacy) < 2e-2, (b, s, nq, nkv, hd)
        assert _rel(lse, lse_legacy) < 1e-4, (b, s, nq, nkv, hd)
    assert native().device_error() == 0
    print("ATTN_FWD_WS_OK")


@opt_in
def test_attention_backward_early_s_order_same_bits(tmp_path):
    """The dK/dV kernel with the next tile's S^T issued before this tile's dK
    (DTB_ATTN_DKDV_EARLY_S=1, read once per process: run in a child process) gives the
    default order's bits."""
    import subprocess
    import sys
    out = tmp_path / "early.pt"
    code = ("import sys; sys.path.insert(0, %r)\n" % os.path.dirname(os.path.dirname(os.path.dirname(
        os.path.abspath(__file__)))) + "from tests.gpu.test_kernels import _attn_bwd_case\n"
        "import torch; torch.save(_attn_bwd_case(), %r)\n" % str(out))
    r = subprocess.run([sys.executable, "-c", code], env=dict(os.environ, DTB_ATTN_DKDV_EARLY_S="1"),
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    early = torch.load(out)
    for a_, b_ in zip(early, _attn_bwd_case()):
        assert torch.equal(a_.to(DEV), b_)


def _attn_bwd_case():
    """Backward of three causal shapes (GQA, several key tiles) from fixed seeds."""
    outs = []
    for (b, s, nq, nkv, hd) in [(1, 1024, 4, 4, 128), (2, 512, 8, 2, 128), (1, 768, 4, 2, 64)]:
        torch.manual_seed(11)
        qkv = _rand(b * s, (nq + 2 * nkv) * hd)
        do = _rand(b * s, nq * hd)
        scale = 1 / math.sqrt(hd)
        o, lse = native().attn_fwd(qkv, b, s, nq, nkv, hd, scale)
        outs.append(native().attn_bwd(do, qkv, o, lse, b, s, nq, nkv, hd, scale))
    assert native().device_error() == 0
    return outs
