"""Megatron tensor parallelism (column/row) with optional sequence parallelism.

Public pieces with the reference's names and semantics
(``src/parallelism/tensor_parallel.py:103-387``):

* the four autograd collectives ``copy_to_tp_region`` (f: identity forward,
  all-reduce backward), ``reduce_from_tp_region`` (g: all-reduce forward),
  ``gather_from_tp_region`` and ``scatter_to_tp_region``;
* ``ColumnParallelLinear`` (weight ``[out/tp, in]``, sharded bias, optional
  ``gather_output``) and ``RowParallelLinear`` (weight ``[out, in/tp]``, full
  bias added once after the reduction, optional input scatter);
* ``apply_tensor_parallelism(model, tp, sequence_parallel=, loss_parallel=)``.

The model plan is the reference's (``:395-501``): ``wq/wk/wv`` and
``gate/up`` column-parallel, ``wo`` and ``down_proj`` row-parallel, embedding,
final norm and head replicated.  It is applied by slicing each rank's shard
out of the full weights (no DTensor), and the blocks call the collectives
below around the fused ops.  Two things the reference declared but could not
run work here:

* ``sequence_parallel``: the residual stream between sub-layers holds
  ``tokens/tp`` rows per rank; column inputs are all-gathered over tokens and
  row outputs reduce-scattered (both fused with their GEMM on GPU), the norms
  run on local tokens and the replicated parameters' gradients are summed over
  the TP group by the sharding engine;
* ``loss_parallel``: vocab-parallel embedding and head with a cross-entropy
  whose max / sum-exp / target-logit terms are reduced over the TP group.

On CUDA with ``fused`` set, the row-parallel GEMM and its all-reduce or
reduce-scatter (+ residual add) run as one kernel over NVLink peer memory
(``csrc/comm.cu``); otherwise the collectives go through ``torch.distributed``
(gloo on CPU; NCCL is the baseline path on GPU).
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Any

import torch
import torch.distributed as dist
import torch.nn as nn
import torch.nn.functional as F

from ..ops.linear import linear


@dataclass
class TPInfo:
    group: dist.ProcessGroup | None
    size: int
    rank: int
    sequence_parallel: bool = False
    fused: bool = False
    comm: Any = None  # symmetric.PeerComm bound to this group when ``fused``


def sp_on(tp: TPInfo | None) -> bool:
    return tp is not None and tp.size > 1 and tp.sequence_parallel


def _size(group: dist.ProcessGroup | None) -> int:
    return dist.get_world_size(group) if group is not None else 1


def _rank(group: dist.ProcessGroup | None) -> int:
    return dist.get_rank(group) if group is not None else 0


# ----------------------------------------------------------------------------
# autograd collectives
# ----------------------------------------------------------------------------
class _CopyToTPRegion(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):  # type: ignore[override]
        ctx.group = group
        return x

    @staticmethod
    def backward(ctx, g):  # type: ignore[override]
        if _size(ctx.group) > 1:
            g = g.contiguous()
            dist.all_reduce(g, group=ctx.group)
        return g, None


class _ReduceFromTPRegion(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):  # type: ignore[override]
        if _size(group) > 1:
            x = x.contiguous().clone()
            dist.all_reduce(x, group=group)
        return x

    @staticmethod
    def backward(ctx, g):  # type: ignore[override]
        return g, None


class _GatherFromTPRegion(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group, dim):  # type: ignore[override]
        ctx.group, ctx.dim = group, dim
        ctx.world, ctx.rank = _size(group), _rank(group)
        if ctx.world == 1:
            return x
        x = x.contiguous()
        parts = [torch.empty_like(x) for _ in range(ctx.world)]
        dist.all_gather(parts, x, group=group)
        return torch.cat(parts, dim=dim)

    @staticmethod
    def backward(ctx, g):  # type: ignore[override]
        if ctx.world == 1:
            return g, None, None
        return g.chunk(ctx.world, dim=ctx.dim)[ctx.rank].contiguous(), None, None


class _ScatterToTPRegion(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group, dim):  # type: ignore[override]
        ctx.group, ctx.dim, ctx.world = group, dim, _size(group)
        if ctx.world == 1:
            return x
        return x.chunk(ctx.world, dim=dim)[_rank(group)].contiguous()

    @staticmethod
    def backward(ctx, g):  # type: ignore[override]
        if ctx.world == 1:
            return g, None, None
        g = g.contiguous()
        parts = [torch.empty_like(g) for _ in range(ctx.world)]
        dist.all_gather(parts, g, group=ctx.group)
        return torch.cat(parts, dim=ctx.dim), None, None


def copy_to_tp_region(x: torch.Tensor, group: dist.ProcessGroup | None) -> torch.Tensor:
    return _CopyToTPRegion.apply(x, group)


def reduce_from_tp_region(x: torch.Tensor, group: dist.ProcessGroup | None) -> torch.Tensor:
    return _ReduceFromTPRegion.apply(x, group)


def gather_from_tp_region(x: torch.Tensor, group: dist.ProcessGroup | None, dim: int = -1) -> torch.Tensor:
    return _GatherFromTPRegion.apply(x, group, dim)


def scatter_to_tp_region(x: torch.Tensor, group: dist.ProcessGroup | None, dim: int = -1) -> torch.Tensor:
    return _ScatterToTPRegion.apply(x, group, dim)


# ---- token-dimension (sequence-parallel) collectives ------------------------
def _all_gather_rows(x: torch.Tensor, tp: TPInfo) -> torch.Tensor:
    if tp.fused and x.is_cuda and tp.comm is not None:
        return tp.comm.all_gather_rows(x)
    out = torch.empty((x.shape[0] * tp.size,) + tuple(x.shape[1:]), device=x.device, dtype=x.dtype)
    if x.is_cuda:
        dist.all_gather_into_tensor(out, x.contiguous(), group=tp.group)
    else:
        parts = list(out.chunk(tp.size, dim=0))
        dist.all_gather(parts, x.contiguous(), group=tp.group)
        out = torch.cat(parts, dim=0)
    return out


def _reduce_scatter_rows(x: torch.Tensor, tp: TPInfo) -> torch.Tensor:
    if tp.fused and x.is_cuda and tp.comm is not None:
        return tp.comm.reduce_scatter_rows(x)
    rows = x.shape[0] // tp.size
    if x.is_cuda:
        out = torch.empty((rows,) + tuple(x.shape[1:]), device=x.device, dtype=x.dtype)
        dist.reduce_scatter_tensor(out, x.contiguous(), group=tp.group)
        return out
    full = x.contiguous().clone()
    dist.all_reduce(full, group=tp.group)
    return full[tp.rank * rows:(tp.rank + 1) * rows].contiguous()


def _fused_ar(tp: TPInfo) -> bool:
    """The NVLink transport's fused all-reduces apply (see ``TPComm.fused_ar``)."""
    return tp.comm is not None and getattr(tp.comm, "fused_ar", True)


def _all_reduce(x: torch.Tensor, tp: TPInfo) -> torch.Tensor:
    if tp.fused and x.is_cuda and _fused_ar(tp):
        return tp.comm.all_reduce(x)
    x = x.contiguous()
    dist.all_reduce(x, group=tp.group)
    return x


class _SeqGather(torch.autograd.Function):
    """All-gather token rows forward, reduce-scatter backward."""

    @staticmethod
    def forward(ctx, x, tp):  # type: ignore[override]
        ctx.tp = tp
        return _all_gather_rows(x, tp)

    @staticmethod
    def backward(ctx, g):  # type: ignore[override]
        return _reduce_scatter_rows(g, ctx.tp), None


class _SeqReduceScatter(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, tp):  # type: ignore[override]
        ctx.tp = tp
        return _reduce_scatter_rows(x, tp)

    @staticmethod
    def backward(ctx, g):  # type: ignore[override]
        return _all_gather_rows(g.contiguous(), ctx.tp), None


class _SeqScatter(torch.autograd.Function):
    """Keep this rank's token rows forward, all-gather backward."""

    @staticmethod
    def forward(ctx, x, tp):  # type: ignore[override]
        ctx.tp = tp
        rows = x.shape[0] // tp.size
        return x[tp.rank * rows:(tp.rank + 1) * rows].contiguous()

    @staticmethod
    def backward(ctx, g):  # type: ignore[override]
        return _all_gather_rows(g.contiguous(), ctx.tp), None


class _AllReduceBwd(torch.autograd.Function):
    """The f operator with the TPInfo transport."""

    @staticmethod
    def forward(ctx, x, tp):  # type: ignore[override]
        ctx.tp = tp
        return x

    @staticmethod
    def backward(ctx, g):  # type: ignore[override]
        return _all_reduce(g.contiguous().clone() if not g.is_cuda else g.contiguous(), ctx.tp), None


class _AllReduceFwd(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, tp):  # type: ignore[override]
        return _all_reduce(x.contiguous().clone() if not x.is_cuda else x.contiguous(), tp)

    @staticmethod
    def backward(ctx, g):  # type: ignore[override]
        return g, None


def reduce_scatter_rows_autograd(x2: torch.Tensor, group: dist.ProcessGroup | None) -> torch.Tensor:
    """Sum over the group and keep this rank's rows (backward: all-gather rows)."""
    tp = TPInfo(group, _size(group), _rank(group), sequence_parallel=True)
    return _SeqReduceScatter.apply(x2, tp)


def sequence_scatter(x2: torch.Tensor, tp: TPInfo | None) -> torch.Tensor:
    assert tp is not None
    return _SeqScatter.apply(x2, tp)


def sequence_slice(t: torch.Tensor, tp: TPInfo | None) -> torch.Tensor:
    assert tp is not None
    rows = t.shape[0] // tp.size
    return t[tp.rank * rows:(tp.rank + 1) * rows]


class SPColumn:
    """Marks a column-parallel layer's transport under sequence parallelism: the layer
    receives this rank's token rows and runs the all-gather inside its GEMM
    (``TPComm.gather_gemm``) and the input gradient's reduce-scatter inside its dgrad
    GEMM (``TPComm.dgrad_reduce_scatter``)."""

    sp = True

    def __init__(self, comm: Any) -> None:
        self.comm = comm


def column_input_fused(x2: torch.Tensor, tp: TPInfo | None, sp_ok: bool = True) -> tuple[torch.Tensor, Any]:
    """Like :func:`column_input`, but when the NVLink transport can fuse the
    input-gradient all-reduce into the column-parallel layer's dgrad GEMM,
    return ``(x2, transport)`` for the layer to do so (no separate f-op).  Under
    sequence parallelism it returns this rank's rows and an :class:`SPColumn`:
    the gather and the gradient's reduce-scatter are fused into the layer's GEMMs."""
    if tp is not None and tp.size > 1 and tp.fused and tp.comm is not None and x2.is_cuda:
        if not tp.sequence_parallel:
            if _fused_ar(tp):
                return x2, tp.comm
            return column_input(x2, tp), None
        if sp_ok and hasattr(tp.comm, "sp_fusable") and tp.comm.sp_fusable(x2):
            return x2, SPColumn(tp.comm)
    return column_input(x2, tp), None


def column_input(x2: torch.Tensor, tp: TPInfo | None) -> torch.Tensor:
    """Input of a column-parallel GEMM: f operator, or token all-gather under SP."""
    if tp is None or tp.size == 1:
        return x2
    if tp.sequence_parallel:
        return _SeqGather.apply(x2, tp)
    return _AllReduceBwd.apply(x2, tp)


def row_output_linear(x2: torch.Tensor, weight: torch.Tensor, residual: torch.Tensor | None,
                      tp: TPInfo | None, *, main_grad: torch.Tensor | None = None,
                      bias: torch.Tensor | None = None) -> torch.Tensor:
    """``reduce(x2 @ W^T) (+ bias) (+ residual)`` for a row-parallel weight."""
    if tp is None or tp.size == 1:
        return linear(x2, weight, bias=bias, residual=residual, main_grad=main_grad)
    if tp.fused and x2.is_cuda and tp.comm is not None and bias is None and (tp.sequence_parallel or _fused_ar(tp)):
        return tp.comm.row_parallel_linear(x2, weight, residual, main_grad)
    y = linear(x2, weight, main_grad=main_grad)
    y = _SeqReduceScatter.apply(y, tp) if tp.sequence_parallel else _AllReduceFwd.apply(y, tp)
    if bias is not None:
        y = y + bias.to(y.dtype)
    return y + residual if residual is not None else y


# ----------------------------------------------------------------------------
# losses split over the TP group
# ----------------------------------------------------------------------------
class _SumOverGroup(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):  # type: ignore[override]
        x = x.clone()
        dist.all_reduce(x, group=group)
        return x

    @staticmethod
    def backward(ctx, g):  # type: ignore[override]
        return g, None


def sequence_parallel_head_ce(h2: torch.Tensor, weight: torch.Tensor, labels: torch.Tensor | None,
                              tp: TPInfo | None, *, main_grad: torch.Tensor | None = None
                              ) -> tuple[torch.Tensor | None, torch.Tensor | None]:
    """Head + CE on this rank's tokens; loss = (sum of local losses) / (global valid count)."""
    from ..ops.loss import lm_head_cross_entropy
    assert tp is not None
    logits, loss = lm_head_cross_entropy(h2, weight, labels, main_grad=main_grad, return_logits=False)
    if labels is None:
        return logits, None
    n_local = (labels != -100).sum().to(torch.float32)
    n_all = n_local.clone()
    dist.all_reduce(n_all, group=tp.group)
    local_sum = torch.nan_to_num(loss.float() * n_local)
    return None, _SumOverGroup.apply(local_sum, tp.group) / n_all


class _VocabParallelCE(torch.autograd.Function):
    """Cross-entropy over logits split by vocabulary over the TP group."""

    @staticmethod
    def forward(ctx, logits, labels, vocab_start, group):  # type: ignore[override]
        lf = logits.float()
        vocab = lf.shape[-1]
        mx = lf.max(dim=-1).values
        dist.all_reduce(mx, op=dist.ReduceOp.MAX, group=group)
        e = torch.exp(lf - mx[:, None])
        se = e.sum(-1)
        dist.all_reduce(se, group=group)
        valid = labels != -100
        local_t = labels - vocab_start
        mine = valid & (local_t >= 0) & (local_t < vocab)
        idx = local_t.clamp(0, vocab - 1)
        tgt = torch.where(mine, lf.gather(1, idx[:, None]).squeeze(1), torch.zeros_like(mx))
        dist.all_reduce(tgt, group=group)
        n = valid.sum().clamp(min=1).float()
        loss = ((torch.log(se) + mx - tgt) * valid).sum() / n
        p = e / se[:, None]
        p[mine, idx[mine]] -= 1.0
        p = p * (valid[:, None].float() / n)
        ctx.save_for_backward(p)
        ctx.dtype = logits.dtype
        return loss

    @staticmethod
    def backward(ctx, g):  # type: ignore[override]
        (p,) = ctx.saved_tensors
        return (p * g).to(ctx.dtype), None, None, None


def vocab_parallel_head_ce(h2: torch.Tensor, weight: torch.Tensor, labels: torch.Tensor | None,
                           tp: TPInfo | None, *, main_grad: torch.Tensor | None = None,
                           vocab_start: int = 0) -> tuple[torch.Tensor | None, torch.Tensor | None]:
    """Column-parallel head (rows = this rank's vocab slice) + vocab-parallel CE."""
    assert tp is not None
    x = column_input(h2, tp)
    if labels is None:
        return linear(x, weight, main_grad=main_grad), None
    # every TP rank holds the full batch's labels; under SP the column input
    # all-gathered the token rows, so the rows cover all tokens as well
    lab = labels.reshape(-1)
    if x.is_cuda and weight.shape[0] % 8 == 0:
        # fused: no logits; the per-row (max, sum exp, target) records cross the TP group
        from ..ops.loss import NcclRowExchange, fused_head_cross_entropy
        comm = tp.comm if (tp.fused and tp.comm is not None) else NcclRowExchange(tp.group)
        return None, fused_head_cross_entropy(x, weight, lab, main_grad=main_grad, vocab_off=vocab_start,
                                              vocab_total=weight.shape[0] * tp.size, comm=comm)
    logits = linear(x, weight, main_grad=main_grad)
    return None, _VocabParallelCE.apply(logits, lab, vocab_start, tp.group)


# ----------------------------------------------------------------------------
# stand-alone parallel linear layers (reference API)
# ----------------------------------------------------------------------------
class ColumnParallelLinear(nn.Module):
    """``y_local = x @ W_local^T + b_local``; ``W_local: [out/tp, in]``."""

    def __init__(self, in_features: int, out_features: int, tp_group: dist.ProcessGroup | None,
                 bias: bool = True, gather_output: bool = False, init_method: Any = None) -> None:
        super().__init__()
        self.tp_group = tp_group
        self.tp_size, self.tp_rank = _size(tp_group), _rank(tp_group)
        if out_features % self.tp_size:
            raise ValueError(
                f"ColumnParallelLinear: out_features={out_features} not divisible by "
                f"tp_size={self.tp_size}.")
        self.in_features, self.out_features = in_features, out_features
        self.out_per_partition = out_features // self.tp_size
        self.gather_output = gather_output
        self.weight = nn.Parameter(torch.empty(self.out_per_partition, in_features))
        self.bias = nn.Parameter(torch.zeros(self.out_per_partition)) if bias else None
        (init_method or (lambda w: nn.init.kaiming_uniform_(w, a=math.sqrt(5))))(self.weight)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        x = copy_to_tp_region(x, self.tp_group)
        y = F.linear(x, self.weight, self.bias)
        return gather_from_tp_region(y, self.tp_group, -1) if self.gather_output else y


class RowParallelLinear(nn.Module):
    """``y = all_reduce(x_local @ W_local^T) + b``; ``W_local: [out, in/tp]``."""

    def __init__(self, in_features: int, out_features: int, tp_group: dist.ProcessGroup | None,
                 bias: bool = True, input_is_parallel: bool = True, init_method: Any = None) -> None:
        super().__init__()
        self.tp_group = tp_group
        self.tp_size, self.tp_rank = _size(tp_group), _rank(tp_group)
        if in_features % self.tp_size:
            raise ValueError(
                f"RowParallelLinear: in_features={in_features} not divisible by "
                f"tp_size={self.tp_size}.")
        self.in_features, self.out_features = in_features, out_features
        self.in_per_partition = in_features // self.tp_size
        self.input_is_parallel = input_is_parallel
        self.weight = nn.Parameter(torch.empty(out_features, self.in_per_partition))
        self.bias = nn.Parameter(torch.zeros(out_features)) if bias else None
        (init_method or (lambda w: nn.init.kaiming_uniform_(w, a=math.sqrt(5))))(self.weight)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if not self.input_is_parallel:
            x = scatter_to_tp_region(x, self.tp_group, -1)
        y = reduce_from_tp_region(F.linear(x, self.weight), self.tp_group)
        return y + self.bias if self.bias is not None else y


# ----------------------------------------------------------------------------
# the model plan
# ----------------------------------------------------------------------------
def _shard_rows(p: nn.Parameter, size: int, rank: int) -> nn.Parameter:
    rows = p.shape[0] // size
    return nn.Parameter(p.detach()[rank * rows:(rank + 1) * rows].clone(), requires_grad=p.requires_grad)


def _shard_cols(p: nn.Parameter, size: int, rank: int) -> nn.Parameter:
    cols = p.shape[1] // size
    return nn.Parameter(p.detach()[:, rank * cols:(rank + 1) * cols].clone(), requires_grad=p.requires_grad)


def _resolve_group(tp: Any) -> dist.ProcessGroup | None:
    if tp is None or isinstance(tp, dist.ProcessGroup):
        return tp
    if hasattr(tp, "get_group"):  # a 1-D DeviceMesh
        return tp.get_group()
    raise TypeError(f"expected a ProcessGroup or 1-D DeviceMesh, got {type(tp)}")


def apply_tensor_parallelism(model: nn.Module, tp_mesh: Any, *, sequence_parallel: bool = False,
                             loss_parallel: bool = False, fused: bool = False) -> nn.Module:
    """Shard every block of ``model`` over the TP group in place.

    Every rank must hold the same full weights beforehand (same seed).  A TP
    group of size 1 leaves the model unchanged.
    """
    group = _resolve_group(tp_mesh)
    size, rank = _size(group), _rank(group)
    if size == 1:
        return model
    info = TPInfo(group, size, rank, sequence_parallel, fused)
    cfg = model.config
    for i, blk in enumerate(model.layers):
        if not (hasattr(blk, "attention") and hasattr(blk, "mlp")):
            raise AttributeError(
                f"block {i} lacks attention/mlp submodules: {list(dict(blk.named_children()))}")
        hd = cfg.head_dim
        for name in ("n_heads", "n_kv_heads"):
            if getattr(cfg, name) % size:
                raise ValueError(f"{name}={getattr(cfg, name)} is not divisible by tp={size}")
        a, m = blk.attention, blk.mlp
        for lin in (a.wq, a.wk, a.wv, m.gate_proj, m.up_proj):
            lin.weight = _shard_rows(lin.weight, size, rank)
            if lin.bias is not None:
                lin.bias = _shard_rows(lin.bias, size, rank)
        for lin in (a.wo, m.down_proj):
            lin.weight = _shard_cols(lin.weight, size, rank)
        assert a.wq.weight.shape[0] % hd == 0
        a.tp = info
        m.tp = info
    model.tp = info
    if loss_parallel:
        from ..models.embeddings import VocabParallelEmbedding
        old = model.tok_embeddings.weight
        emb = VocabParallelEmbedding(cfg.vocab_size, cfg.d_model, group)
        emb.weight = _shard_rows(old, size, rank)
        model.tok_embeddings = emb
        if cfg.tie_embeddings:
            model.lm_head.weight = emb.weight
        else:
            model.lm_head.weight = _shard_rows(model.lm_head.weight, size, rank)
    return model


def tp_param_kind(fqn: str, model: nn.Module) -> str:
    """``"row"`` (dim-0 split), ``"col"`` (dim-1 split) or ``"rep"`` (replicated) under TP."""
    tp = getattr(model, "tp", None)
    if tp is None or tp.size == 1:
        return "rep"
    if fqn.endswith(("attention.wq.weight", "attention.wk.weight", "attention.wv.weight",
                     "mlp.gate_proj.weight", "mlp.up_proj.weight", "attention.wq.bias",
                     "attention.wk.bias", "attention.wv.bias", "mlp.gate_proj.bias",
                     "mlp.up_proj.bias")):
        return "row"
    if fqn.endswith(("attention.wo.weight", "mlp.down_proj.weight")):
        return "col"
    from ..models.embeddings import VocabParallelEmbedding
    if isinstance(getattr(model, "tok_embeddings", None), VocabParallelEmbedding) and fqn in (
            "tok_embeddings.weight", "lm_head.weight"):
        return "row"
    return "rep"
