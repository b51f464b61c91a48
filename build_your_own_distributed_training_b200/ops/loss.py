"""LM head + cross-entropy (mean over labels != -100).

Reference: ``src/model/transformer.py:184-191`` (cuBLAS GEMM to logits, then
``F.cross_entropy``) and, split over the vocabulary, ``loss_parallel`` at
``src/parallelism/tensor_parallel.py:396-400``.

CUDA path, fused (``lm_head_cross_entropy(..., return_logits=False)``, what
training uses): no ``[tokens, vocab]`` tensor is ever written.

* forward: the tcgen05 head GEMM's epilogue reduces each 128/256-column tile of
  the logits to a per-row (max, sum exp) pair and picks out the label's logit
  (``gemm_ce_stats``); ``ce_stats_reduce`` merges the column blocks into the
  row's log-sum-exp, and ``ce_loss_finish`` takes the fixed-order mean and the
  device scalar ``1 / n_valid``.  With the vocabulary split over the TP group,
  each rank's (max, sum, target) rows are merged through the TP symmetric heap
  (``ce_peer_combine``, rank order, identical bits on every rank).
* backward: per vocabulary chunk of ``CHUNK`` columns, the head GEMM is
  recomputed with an epilogue that writes the bf16 logit gradient
  ``(softmax - onehot) * dloss / n_valid`` for that chunk only
  (``gemm_ce_grad``); the chunk feeds the input-gradient GEMM (fp32
  accumulation across chunks, bf16 out of the last) and the weight-gradient
  GEMM into the chunk's rows of ``main_grad``.

The unfused path (``return_logits=True``) writes fp32 logits and runs one CE
kernel per row; it is kept for callers that want the logits.
"""

from __future__ import annotations

import os

import torch
import torch.nn.functional as F

from . import gemm, grad_state
from ._ext import native

IGNORE = -100
CHUNK = int(os.environ.get("DTB_CE_CHUNK", "8192"))  # vocabulary columns per backward chunk


class _HeadCEFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, w, labels, main_grad, keep_logits):  # type: ignore[override]
        logits = gemm.mm_nt(h, w, out_dtype=torch.float32)
        loss, dlogits = native().cross_entropy_fwd(logits, labels, IGNORE)
        ctx.save_for_backward(h, w, dlogits)
        ctx.main_grad = main_grad
        return loss, (logits if keep_logits else None)

    @staticmethod
    def backward(ctx, dloss, _dlogits_unused):  # type: ignore[override]
        h, w, dlogits = ctx.saved_tensors
        alpha = dloss.reshape(1).float().contiguous()
        dh = gemm.mm_nn(dlogits, w, alpha=alpha)
        if ctx.main_grad is not None:
            gemm.mm_tn_into_grad(dlogits, h, ctx.main_grad, w.shape, alpha=alpha)
            dw = None
        elif w.requires_grad:
            dw = gemm.mm_tn(dlogits, h, alpha=alpha).to(w.dtype)
        else:
            dw = None
        return dh, dw, None, None, None


def fused_ce_forward(h: torch.Tensor, w: torch.Tensor, labels: torch.Tensor, vocab_off: int, vocab_total: int,
                     comm=None) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Loss, per-row log-sum-exp and ``1 / n_valid`` of ``CE(h @ w^T)`` without the logits.

    ``w`` holds vocabulary rows ``[vocab_off, vocab_off + w.shape[0])`` of ``vocab_total``;
    with ``comm`` the other rows live on the other ranks of a TP group, and ``comm`` moves
    each rank's 16-byte (max, sum exp, target logit) row records: the NVLink transport's
    ``TPComm`` (symmetric heap + device barrier) or :class:`NcclRowExchange`.
    """
    M, V = h.shape[0], w.shape[0]
    nblk = native().gemm_ce_blocks(V)
    stats = torch.empty(M, 2 * nblk, device=h.device, dtype=torch.float32)
    tgt = torch.empty(M, device=h.device, dtype=torch.float32)
    native().gemm_ce_stats(h, w, labels, stats, tgt, vocab_off, vocab_total, IGNORE)
    lse = torch.empty(M, device=h.device, dtype=torch.float32)
    rows = torch.empty(M, device=h.device, dtype=torch.float32)
    if comm is None:
        native().ce_stats_reduce(stats, tgt, labels, vocab_off, V, vocab_total, IGNORE, lse, rows, None)
    else:
        off, xchg = comm.exchange_rows(M, 16)
        native().ce_stats_reduce(stats, tgt, labels, vocab_off, V, vocab_total, IGNORE, lse, rows, xchg)
        bases, off = comm.exchange_publish(off, xchg)
        native().ce_peer_combine(bases, off, labels, vocab_total, IGNORE, lse, rows)
    loss = torch.empty((), device=h.device, dtype=torch.float32)
    inv_n = torch.empty(1, device=h.device, dtype=torch.float32)
    native().ce_loss_finish(rows, labels, vocab_total, IGNORE, loss, inv_n)
    return loss, lse, inv_n


def fused_ce_backward(h: torch.Tensor, w: torch.Tensor, labels: torch.Tensor, lse: torch.Tensor,
                      inv_n: torch.Tensor, dloss: torch.Tensor, vocab_off: int, vocab_total: int,
                      main_grad: torch.Tensor | None, chunk: int = CHUNK
                      ) -> tuple[torch.Tensor, torch.Tensor | None]:
    """``(dh, dw)`` of the fused loss; ``dw`` is ``None`` when it went into ``main_grad``."""
    M, V = h.shape[0], w.shape[0]
    chunk = max(256, (chunk // 256) * 256)
    alpha = dloss.reshape(1).float().contiguous()
    store = grad_state.take_fresh(main_grad) if main_grad is not None else True
    gview = main_grad.view(w.shape) if main_grad is not None else None
    dw = None if main_grad is not None else torch.empty(w.shape, device=w.device, dtype=torch.float32)
    n_chunks = -(-V // chunk)
    dh = torch.empty(M, w.shape[1], device=h.device, dtype=h.dtype)
    acc = torch.empty(M, w.shape[1], device=h.device, dtype=torch.float32) if n_chunks > 1 else None
    dl_buf = torch.empty(M * min(chunk, V), device=h.device, dtype=h.dtype)
    for ci in range(n_chunks):
        c0, c1 = ci * chunk, min(V, (ci + 1) * chunk)
        wc = w[c0:c1]
        dl = dl_buf[:M * (c1 - c0)].view(M, c1 - c0)
        native().gemm_ce_grad(h, wc, labels, lse, alpha, inv_n, dl, vocab_off + c0, vocab_total, IGNORE)
        # input gradient: sum over chunks of dl_c @ w_c, fp32 between chunks, bf16 out of the last
        if n_chunks == 1:
            gemm.mm_nn(dl, wc, out=dh)
        elif ci == 0:
            native().gemm(dl, wc, acc, False, True, gemm.EPI_STORE, None, None, None, None, None, 0, 0)
        elif ci < n_chunks - 1:
            native().gemm(dl, wc, acc, False, True, gemm.EPI_ACC_F32, None, None, None, None, None, 0, 0)
        else:
            native().gemm(dl, wc, dh, False, True, gemm.EPI_ACC_BF16OUT, acc, None, None, None, None, 0, 0)
        # weight gradient of the chunk's rows
        if gview is not None:
            gemm.mm_tn_acc(dl, h, gview[c0:c1], store=store)
        else:
            gemm.mm_tn_acc(dl, h, dw[c0:c1], store=True)
    return dh, (dw.to(w.dtype) if dw is not None else None)


class NcclRowExchange:
    """Row-record exchange for the vocabulary-parallel CE over a process group (NCCL),
    used when the NVLink transport is off: an all-gather, then the same combine kernel
    reading the gathered copies in rank order."""

    def __init__(self, group) -> None:
        self.group = group
        self._keep: list[torch.Tensor] = []

    def exchange_rows(self, rows: int, row_bytes: int) -> tuple[int, torch.Tensor]:
        return 0, torch.empty(rows * row_bytes // 4, device="cuda", dtype=torch.float32)

    def exchange_publish(self, off: int, rows: torch.Tensor) -> tuple[list[int], int]:
        import torch.distributed as dist
        n = dist.get_world_size(self.group)
        gathered = torch.empty(n * rows.numel(), device=rows.device, dtype=rows.dtype)
        dist.all_gather_into_tensor(gathered, rows, group=self.group)
        self._keep = [gathered, rows]  # alive until the combine kernel has run (stream order)
        step = rows.numel() * rows.element_size()
        return [gathered.data_ptr() + r * step for r in range(n)], 0


class _FusedHeadCEFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, w, labels, main_grad, vocab_off, vocab_total, comm):  # type: ignore[override]
        loss, lse, inv_n = fused_ce_forward(h, w, labels, vocab_off, vocab_total, comm)
        ctx.save_for_backward(h, w, labels, lse, inv_n)
        ctx.main_grad = main_grad
        ctx.vocab = (vocab_off, vocab_total)
        ctx.w_grad = w.requires_grad
        return loss

    @staticmethod
    def backward(ctx, dloss):  # type: ignore[override]
        h, w, labels, lse, inv_n = ctx.saved_tensors
        dh, dw = fused_ce_backward(h, w, labels, lse, inv_n, dloss, ctx.vocab[0], ctx.vocab[1], ctx.main_grad)
        return dh, (dw if ctx.w_grad else None), None, None, None, None, None


def fused_head_cross_entropy(h: torch.Tensor, weight: torch.Tensor, labels: torch.Tensor, *,
                             main_grad: torch.Tensor | None = None, vocab_off: int = 0,
                             vocab_total: int | None = None, comm=None) -> torch.Tensor:
    """Mean CE of ``h @ weight^T`` over labels != -100, never materialising the logits (CUDA)."""
    vt = weight.shape[0] if vocab_total is None else vocab_total
    return _FusedHeadCEFn.apply(h.contiguous(), weight, labels.reshape(-1).contiguous(), main_grad,
                                int(vocab_off), int(vt), comm)


def lm_head_cross_entropy(h: torch.Tensor, weight: torch.Tensor, labels: torch.Tensor | None, *,
                          main_grad: torch.Tensor | None = None, return_logits: bool = True
                          ) -> tuple[torch.Tensor | None, torch.Tensor | None]:
    """Returns ``(logits or None, loss or None)`` for ``h: [M, d]``, ``labels: [M]``."""
    if not h.is_cuda or labels is None:
        from .linear import linear
        logits = linear(h, weight, main_grad=main_grad)
        loss = None
        if labels is not None:
            loss = F.cross_entropy(logits.float(), labels.reshape(-1), ignore_index=IGNORE)
        return logits, loss
    if not return_logits and weight.shape[0] % 8 == 0:
        return None, fused_head_cross_entropy(h, weight, labels, main_grad=main_grad)
    loss, logits = _HeadCEFn.apply(h.contiguous(), weight, labels.reshape(-1).contiguous(),
                                   main_grad, return_logits)
    return logits, loss
