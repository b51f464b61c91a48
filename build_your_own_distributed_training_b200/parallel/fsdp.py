"""ZeRO-3 sharding engine over flat per-block buffers (replaces FSDP1).

Reference behaviour reproduced (``src/parallelism/fsdp_utils.py:94-227``,
``src/training/loop.py:74-84``, ``docs/ARCHITECTURE.md:71-98``):

* one sharding unit per ``TransformerBlock`` plus a root unit with the
  remaining parameters (embedding, final norm, head; a tied weight counts once);
* ``FULL_SHARD``: parameters live as 1/dp shards; a unit's full parameters are
  gathered before its forward, dropped after it and gathered again before its
  backward; ``SHARD_GRAD_OP`` keeps them gathered from forward to backward;
  ``NO_SHARD`` keeps full replicas and all-reduces gradients; ``HYBRID_SHARD``
  shards within a node and replicates across nodes (on one node it is
  ``FULL_SHARD``);
* compute parameters in ``param_dtype`` (bf16), gradients reduced in fp32 and
  averaged over dp, fp32 master weights and optimizer state on the shard;
* ``no_sync()``: gradients accumulate locally; the reduce-scatter runs only on
  the synchronising micro-step;
* forward prefetch of the next unit and backward prefetch of the previous one
  on a side stream, at most two gathered blocks alive with
  ``limit_all_gathers``.

Layout.  A unit's parameters are packed into one flat buffer in the order
[TP-sharded matrices | replicated matrices | vectors], each entry aligned to
64 elements.  Inside a block the matrices are ``wq, wk, wv, wo, gate, up,
down``, so ``[wq; wk; wv]`` and ``[gate; up]`` are contiguous and the fused
QKV and SwiGLU GEMMs take them as single weights without a copy.  The
category boundaries let the optimizer apply weight decay to matrices only and
let the gradient norm count TP-replicated entries once.

Gradients.  Every unit owns a persistent fp32 gradient buffer of its full
size; each parameter gets a ``main_grad`` view into it and the kernels'
weight-gradient GEMMs accumulate there directly (no per-parameter gradient
tensors).  Micro-step accumulation is that same in-place add.  After the
synchronising backward of a unit its buffer is reduce-scattered (mean over dp)
into the unit's fp32 gradient shard.

Collectives go through ``comm``: :class:`TorchComm` (``torch.distributed``;
gloo on CPU, NCCL as the GPU baseline) or ``symmetric.PeerComm`` (this
package's NVLink peer-memory kernels).
"""

from __future__ import annotations

import contextlib
import warnings
from dataclasses import dataclass, field
from typing import Any, Iterable

import torch
import torch.distributed as dist
import torch.nn as nn

from ..config import ParallelConfig
from ..observability import nvtx
from ..ops import grad_state
from ..utils.dtype import build_mixed_precision
from .tensor_parallel import tp_param_kind

ALIGN = 64


def _align(n: int, a: int = ALIGN) -> int:
    return -(-n // a) * a


@dataclass
class Entry:
    fqn: str
    param: nn.Parameter
    shape: torch.Size
    numel: int
    offset: int
    tp_kind: str      # "row" | "col" | "rep"
    decay: bool


@dataclass
class FlatUnit:
    index: int
    name: str
    module: nn.Module
    entries: list[Entry]
    numel: int                    # padded flat size P
    shard_numel: int              # S = P / shard_world
    tp_end: int                   # [0, tp_end): TP-sharded entries
    decay_end: int                # [0, decay_end): matrices (weight decay applies)
    master: torch.Tensor | None = None       # fp32 [S]
    param_shard: torch.Tensor | None = None  # param_dtype [S]
    grad: torch.Tensor | None = None         # fp32 [P]
    grad_shard: torch.Tensor | None = None   # fp32 [S]
    gathered: torch.Tensor | None = None     # param_dtype [P] (persistent or slot)
    slot: int = -1
    fresh: Any = None                        # FreshSet over ``grad`` (lazily zeroed slices)
    extras: dict = field(default_factory=dict)

    def shard_range(self, rank: int) -> tuple[int, int]:
        return rank * self.shard_numel, (rank + 1) * self.shard_numel


class TorchComm:
    """Unit collectives through ``torch.distributed`` (gloo on CPU, NCCL on GPU)."""

    name = "torch"

    def __init__(self, group: dist.ProcessGroup | None, size: int, rank: int,
                 replicate_group: dist.ProcessGroup | None = None, replicate_size: int = 1) -> None:
        self.group, self.size, self.rank = group, size, rank
        self.rgroup, self.rsize = replicate_group, replicate_size

    def all_gather(self, out_full: torch.Tensor, shard: torch.Tensor) -> None:
        if self.size == 1:
            out_full.copy_(shard)
            return
        if shard.is_cuda:
            dist.all_gather_into_tensor(out_full, shard, group=self.group)
        else:
            dist.all_gather(list(out_full.chunk(self.size)), shard, group=self.group)

    def reduce_scatter_mean(self, out_shard: torch.Tensor, full: torch.Tensor, world: int) -> None:
        if self.size == 1:
            if out_shard.data_ptr() != full.data_ptr():
                out_shard.copy_(full)
        elif full.is_cuda:
            dist.reduce_scatter_tensor(out_shard, full, group=self.group)
        else:
            tmp = full.clone()
            dist.all_reduce(tmp, group=self.group)
            out_shard.copy_(tmp.chunk(self.size)[self.rank])
        if self.rsize > 1:
            dist.all_reduce(out_shard, group=self.rgroup)
        if world != 1:
            out_shard.div_(world)

    def all_reduce_sum(self, t: torch.Tensor, group: dist.ProcessGroup | None) -> None:
        dist.all_reduce(t, group=group)

    def barrier(self) -> None:
        pass


class FullyShardedModel(nn.Module):
    """The sharded model; ``forward`` has the wrapped model's signature."""

    def __init__(self, module: nn.Module, ctx: Any, cfg: ParallelConfig,
                 layer_cls: Iterable[type[nn.Module]], *, comm: Any = None,
                 device: torch.device | None = None) -> None:
        super().__init__()
        self.module = module
        self.ctx = ctx
        self.cfg = cfg
        self.policy = build_mixed_precision(cfg)
        self.device = device or (ctx.device if ctx is not None else torch.device("cpu"))
        if self.device.type == "cuda" and self.policy.param_dtype != torch.bfloat16:
            raise ValueError(
                f"parallel.param_dtype={cfg.param_dtype}: the CUDA kernels compute in bf16 (fp32 master "
                "weights, fp32 gradient reduction); set parallel.param_dtype: bfloat16 for GPU runs "
                "(float32 compute runs on the CPU/gloo path only)")
        dims = ctx.dims if ctx is not None else None
        self.dp_size = dims.dp_size if dims else 1
        self.dp_rank = dims.dp_rank if dims else 0
        self.tp_size = dims.tp_size if dims else 1
        self.dp_group = ctx.dp_group if ctx is not None else None
        self.tp_group = ctx.tp_group if ctx is not None else None
        self.strategy = cfg.sharding_strategy
        self.shard_world, self.shard_rank = self.dp_size, self.dp_rank
        rgroup, rsize = None, 1
        if self.strategy == "NO_SHARD":
            self.shard_world, self.shard_rank = 1, 0
        elif self.strategy == "HYBRID_SHARD":
            self.shard_world, self.shard_rank, sgroup, rgroup, rsize = _hybrid_groups(ctx)
        self.comm = comm or TorchComm(
            None if self.strategy == "NO_SHARD" else (
                sgroup if self.strategy == "HYBRID_SHARD" else self.dp_group),
            self.shard_world, self.shard_rank, rgroup if self.strategy != "NO_SHARD" else self.dp_group,
            rsize if self.strategy != "NO_SHARD" else self.dp_size)
        self.replication = self.dp_size // self.shard_world
        self._sync = True
        self._layer_cls = tuple(layer_cls)
        self.units: list[FlatUnit] = []
        self.blocks: list[nn.Module] = [m for m in module.modules() if isinstance(m, self._layer_cls)]
        self._build_units()
        self._alloc()
        self._install_hooks()
        self._is_cuda = self.device.type == "cuda"
        self._comm_stream = torch.cuda.Stream(device=self.device) if self._is_cuda else None
        self._ready: dict[int, Any] = {}
        self._slot_owner: dict[int, int] = {}
        self._rs_pending: list[Any] = []
        self._bwd_started = False
        # transports whose reduce-scatter also yields the gradient-norm partials
        # (per unit, per block; zero where a unit uses fewer blocks)
        self._norm_parts: torch.Tensor | None = None
        self._norm_fresh = [False] * len(self.units)
        if getattr(self.comm, "norm_partials", False) and self.units and self.replication == 1:
            nb = max(self.comm.norm_partial_blocks(u.shard_numel) for u in self.units)
            self._norm_parts = torch.zeros(len(self.units), nb, device=self.device, dtype=torch.float32)
        # otherwise: each unit's sums of squares [plain part, TP-replicated part] of its
        # gradient shard, taken right after the unit's reduction (on CUDA on the communication
        # stream, so the pass over the gradients overlaps the rest of the backward instead of
        # following it); the same kernels and summation order as a pass after the backward
        self._unit_ss: torch.Tensor | None = None
        self._ss_fresh = [False] * len(self.units)
        if self.units and self._norm_parts is None:
            self._unit_ss = torch.zeros(len(self.units), 2, device=self.device, dtype=torch.float32)
        self._gather_all_root()

    # ------------------------------------------------------------------ build
    def _build_units(self) -> None:
        seen: set[int] = set()
        owned: dict[int, int] = {}
        groups: list[tuple[str, nn.Module, list[tuple[str, nn.Parameter]]]] = []
        for bi, blk in enumerate(self.blocks):
            plist = []
            prefix = _prefix_of(self.module, blk)
            for n, p in blk.named_parameters():
                if id(p) in seen:
                    continue
                seen.add(id(p))
                owned[id(p)] = bi
                plist.append((f"{prefix}{n}", p))
            groups.append((prefix.rstrip("."), blk, plist))
        root = []
        for n, p in self.module.named_parameters():
            if id(p) not in seen:
                seen.add(id(p))
                root.append((n, p))
        groups.append(("<root>", self.module, root))
        for ui, (name, mod, plist) in enumerate(groups):
            cats: list[list[tuple[str, nn.Parameter, str]]] = [[], [], []]
            for fqn, p in plist:
                kind = tp_param_kind(fqn, self.module)
                if p.dim() >= 2:
                    cats[0 if kind != "rep" else 1].append((fqn, p, kind))
                else:
                    cats[2].append((fqn, p, kind))
            entries: list[Entry] = []
            off = 0
            bounds = []
            for ci, cat in enumerate(cats):
                for fqn, p, kind in cat:
                    entries.append(Entry(fqn, p, p.shape, p.numel(), off, kind,
                                         decay=(ci < 2)))
                    off = _align(off + p.numel())
                bounds.append(off)
            total = _align(max(off, 1), ALIGN * self.shard_world)
            self.units.append(FlatUnit(ui, name, mod, entries, total, total // self.shard_world,
                                       tp_end=bounds[0], decay_end=bounds[1]))

    def _alloc(self) -> None:
        dev = self.device
        pdt = self.policy.param_dtype
        # buffers peers read (parameter shards, gradient buffers) go into the
        # transport's symmetric heap when it has one
        heap_views: list[torch.Tensor] = []
        if hasattr(self.comm, "alloc_many"):
            specs = []
            for u in self.units:
                specs += [(u.shard_numel, pdt), (u.numel, torch.float32)]
            heap_views = self.comm.alloc_many(specs)
        for ui, u in enumerate(self.units):
            full = torch.zeros(u.numel, dtype=torch.float32)
            for e in u.entries:
                full[e.offset:e.offset + e.numel] = e.param.detach().reshape(-1).float().cpu()
            lo, hi = u.shard_range(self.shard_rank)
            u.master = full[lo:hi].clone().to(dev)
            if heap_views:
                u.param_shard, u.grad = heap_views[2 * ui], heap_views[2 * ui + 1]
            else:
                u.param_shard = torch.empty(u.shard_numel, dtype=pdt, device=dev)
                u.grad = torch.empty(u.numel, dtype=torch.float32, device=dev)
            u.param_shard.copy_(u.master.to(pdt))
            u.grad.zero_()  # padding stays zero for good; parameter slices go lazy from here
            u.fresh = grad_state.FreshSet(u.grad)
            # unsharded units reduce in place: the gradient shard is the gradient buffer
            u.grad_shard = u.grad if self.shard_world == 1 else torch.zeros(u.shard_numel, dtype=torch.float32,
                                                                            device=dev)
        n_slots = 2 if self.cfg.limit_all_gathers else 3
        block_units = self.units[:-1]
        persistent = self.strategy in ("NO_SHARD", "SHARD_GRAD_OP") or self.shard_world == 1
        self._slots: list[torch.Tensor] = []
        if block_units and not persistent:
            self._slots = [torch.empty(block_units[0].numel, dtype=pdt, device=dev) for _ in range(n_slots)]
        for u in self.units:
            if self.shard_world == 1:
                u.gathered = u.param_shard  # the shard is the whole unit: gathering is a no-op
            elif u is self.units[-1] or persistent or not self._slots:
                u.gathered = torch.empty(u.numel, dtype=pdt, device=dev)
            else:
                if u.numel != block_units[0].numel:  # heterogeneous blocks: own buffer
                    u.gathered = torch.empty(u.numel, dtype=pdt, device=dev)
                else:
                    u.slot = u.index % len(self._slots)
                    u.gathered = self._slots[u.slot]
            self._bind(u)

    def _bind(self, u: FlatUnit) -> None:
        assert u.gathered is not None and u.grad is not None
        for e in u.entries:
            e.param.data = u.gathered[e.offset:e.offset + e.numel].view(e.shape)
            e.param.main_grad = grad_state.tag(  # type: ignore[attr-defined]
                u.grad[e.offset:e.offset + e.numel].view(e.shape), u.fresh, e.offset)

    # ------------------------------------------------------------------ hooks
    def _install_hooks(self) -> None:
        for bi, blk in enumerate(self.blocks):
            blk.register_forward_pre_hook(self._make_pre_fwd(bi))
            blk.register_forward_hook(self._make_post_fwd(bi))

    def _make_pre_fwd(self, bi: int):
        def hook(_mod, args):
            in_bwd = _in_backward()
            nvtx.push(f"block{bi}.{'recompute' if in_bwd else 'fwd'}")
            if torch.is_grad_enabled() and not in_bwd and args and isinstance(args[0], torch.Tensor) \
                    and args[0].requires_grad:
                args[0].register_hook(lambda g, bi=bi: self._post_backward(bi))
            self._ensure(bi)
            if self.cfg.forward_prefetch and not in_bwd and bi + 1 < len(self.blocks):
                self._prefetch(bi + 1)
        return hook

    def _make_post_fwd(self, bi: int):
        def hook(_mod, _args, out):
            if torch.is_grad_enabled() and not _in_backward() and isinstance(out, torch.Tensor) \
                    and out.requires_grad:
                out.register_hook(lambda g, bi=bi: self._pre_backward(bi))
            nvtx.pop()
            return out
        return hook

    def _pre_backward(self, bi: int) -> None:
        nvtx.push(f"block{bi}.bwd")
        if not self._bwd_started:
            self._bwd_started = True
            # gradients change from here: the norm terms of an earlier reduction are stale
            self._norm_fresh = [False] * len(self.units)
            self._ss_fresh = [False] * len(self.units)
            torch.autograd.Variable._execution_engine.queue_callback(self._finish_backward)
        self._ensure(bi)
        # BACKWARD_PRE: gather the previous block while this one computes its gradients
        if bi - 1 >= 0 and self.cfg.backward_prefetch == "BACKWARD_PRE":
            self._prefetch(bi - 1)

    def _post_backward(self, bi: int) -> None:
        nvtx.pop()
        # BACKWARD_POST: gather the previous block once this one's gradients are done
        # (less overlap, one gathered block fewer alive during the gradient GEMMs)
        if bi - 1 >= 0 and self.cfg.backward_prefetch == "BACKWARD_POST":
            self._prefetch(bi - 1)
        u = self.units[bi]
        if self._sync:
            self._reduce_scatter(u)

    def _finish_backward(self) -> None:
        self._bwd_started = False
        if self._sync:
            self._reduce_scatter(self.units[-1])
            self.wait_reduce()

    # ------------------------------------------------------------ gathering
    def _gather_into(self, u: FlatUnit) -> None:
        assert u.gathered is not None and u.param_shard is not None
        if u.gathered is u.param_shard:
            return
        self.comm.all_gather(u.gathered, u.param_shard)

    def _prefetch(self, bi: int) -> None:
        u = self.units[bi]
        if u.slot < 0:
            return
        if self._slot_owner.get(u.slot) == bi or bi in self._ready:
            return
        if not self._is_cuda:
            return  # gathered synchronously in _ensure
        s = self._comm_stream
        # everything enqueued so far includes the last reader of this slot
        # (the previous block's forward, or the next block's backward)
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            self._gather_into(u)
            ev = torch.cuda.Event()
            ev.record(s)
        self._slot_owner[u.slot] = bi
        self._ready[bi] = ev

    def _ensure(self, bi: int) -> None:
        u = self.units[bi]
        if u.slot < 0:
            return
        if bi in self._ready:
            torch.cuda.current_stream().wait_event(self._ready.pop(bi))
            return
        if self._slot_owner.get(u.slot) == bi:
            return
        self._gather_into(u)
        self._slot_owner[u.slot] = bi

    def _gather_all_root(self) -> None:
        """(Re)gather every persistent buffer from the shards (after init / optimizer step)."""
        self.comm.barrier()
        self._ready.clear()
        self._slot_owner.clear()
        for u in self.units:
            if u.slot < 0:
                self._gather_into(u)

    def after_optimizer_step(self) -> None:
        """New shards are in place: refresh gathered parameters."""
        self._gather_all_root()

    # ------------------------------------------------------------ reduction
    def _reduce_scatter(self, u: FlatUnit) -> None:
        assert u.grad is not None and u.grad_shard is not None
        u.fresh.flush()  # slices no kernel wrote this step are zero gradients
        if self._is_cuda:
            s = self._comm_stream
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                self._rs_body(u)
        else:
            self._rs_body(u)

    def _rs_body(self, u: FlatUnit) -> None:
        if self.tp_size > 1 and getattr(getattr(self.module, "tp", None), "sequence_parallel", False) \
                and u.tp_end < u.numel:
            # under sequence parallelism replicated parameters got partial grads per TP rank
            rep = u.grad[u.tp_end:]
            self.comm.all_reduce_sum(rep, self.tp_group) if not hasattr(self.comm, "tp_all_reduce") \
                else self.comm.tp_all_reduce(rep)
        if self._norm_parts is not None:
            lo, hi = u.shard_range(self.shard_rank)
            split = min(max(u.tp_end - lo, 0), hi - lo)  # shard-local start of the TP-replicated entries
            self.comm.reduce_scatter_mean(u.grad_shard, u.grad, self.dp_size, part=self._norm_parts[u.index],
                                          split=split, rep_w=1.0 / self.tp_size)
            self._norm_fresh[u.index] = True
        else:
            self.comm.reduce_scatter_mean(u.grad_shard, u.grad, self.dp_size)
            if self._unit_ss is not None:
                for k, (a, b) in enumerate(self._norm_segments(u)):
                    if b > a:
                        self._unit_ss[u.index, k].copy_(_sumsq(u.grad_shard[a:b]))
                self._ss_fresh[u.index] = True

    def _norm_segments(self, u: FlatUnit) -> tuple[tuple[int, int], tuple[int, int]]:
        """Shard-local ranges of the unit's plain and TP-replicated gradient entries."""
        lo, hi = u.shard_range(self.shard_rank)
        a, b = _clip(0, u.tp_end, lo, hi)
        c, d = _clip(u.tp_end, u.numel, lo, hi)
        return (a - lo, b - lo), (c - lo, d - lo)

    def wait_reduce(self) -> None:
        if self._is_cuda:
            torch.cuda.current_stream().wait_stream(self._comm_stream)

    @contextlib.contextmanager
    def no_sync(self):
        prev = self._sync
        self._sync = False
        try:
            yield
        finally:
            self._sync = prev

    def zero_grad_buffers(self) -> None:
        """Logically zero every gradient: slices become fresh, the first writer overwrites them."""
        self._norm_fresh = [False] * len(self.units)
        self._ss_fresh = [False] * len(self.units)
        for u in self.units:
            u.fresh.mark([(e.offset, e.numel) for e in u.entries])

    # ------------------------------------------------------------ forward
    def forward(self, *args: Any, **kwargs: Any) -> Any:
        return self.module(*args, **kwargs)

    # ------------------------------------------------------------ queries
    def shard_views(self) -> list[tuple[FlatUnit, int, int]]:
        return [(u, *u.shard_range(self.shard_rank)) for u in self.units]

    def grad_norm_sq_local(self) -> torch.Tensor:
        """Sum of g^2 over this rank's gradient shards; TP-replicated entries weighted 1/tp.

        When this step's reduce-scatters left their per-block partials (NVLink transport),
        this is one fixed-order sum over them; otherwise the per-unit terms taken after each
        unit's reduction (or, if a unit was not reduced since the backward began, a pass over
        its shard) summed in unit order."""
        if self._norm_parts is not None and all(self._norm_fresh):
            from ..ops._ext import native
            return native().sum_small(self._norm_parts)
        ready = self._unit_ss is not None and all(self._ss_fresh)
        tot = torch.zeros((), dtype=torch.float32, device=self.device)
        for u in self.units:
            (a, b), (c, d) = self._norm_segments(u)
            if b > a:
                tot = tot + (self._unit_ss[u.index, 0] if ready else _sumsq(u.grad_shard[a:b]))
            if d > c:
                tot = tot + (self._unit_ss[u.index, 1] if ready else _sumsq(u.grad_shard[c:d])) / self.tp_size
        # NO_SHARD / HYBRID_SHARD hold the same averaged shard on several dp ranks
        return tot / self.replication

    def unsharded_numel(self) -> int:
        return sum(e.numel for u in self.units for e in u.entries)

    def full_flat_params(self, u: FlatUnit) -> torch.Tensor:
        """fp32 full flat parameters of one unit (all-gathered master)."""
        assert u.master is not None
        if self.shard_world == 1:
            return u.master.clone()
        out = torch.empty(u.numel, dtype=torch.float32, device=u.master.device)
        if u.master.is_cuda:
            dist.all_gather_into_tensor(out, u.master, group=self.comm.group)
        else:
            dist.all_gather(list(out.chunk(self.shard_world)), u.master, group=self.comm.group)
        return out


def _in_backward() -> bool:
    """True while the autograd engine runs (e.g. an activation-checkpoint recompute)."""
    return torch._C._current_graph_task_id() != -1


def _sumsq(t: torch.Tensor) -> torch.Tensor:
    if t.is_cuda:
        from ..ops._ext import native
        return native().sumsq(t)
    return t.double().pow(2).sum().float()


def _clip(a: int, b: int, lo: int, hi: int) -> tuple[int, int]:
    return max(a, lo), min(b, hi)


def _prefix_of(root: nn.Module, sub: nn.Module) -> str:
    for name, m in root.named_modules():
        if m is sub:
            return f"{name}." if name else ""
    raise ValueError("module not found under root")


def _hybrid_groups(ctx: Any) -> tuple[int, int, Any, Any, int]:
    """Shard inside a node, replicate across nodes (dp axis split by node)."""
    env = ctx.env
    tp = ctx.dims.tp_size
    per_node_dp = max(1, env.local_world_size // tp)
    dp, dpr = ctx.dims.dp_size, ctx.dims.dp_rank
    if per_node_dp >= dp:
        return dp, dpr, ctx.dp_group, None, 1
    nodes = dp // per_node_dp
    mesh = ctx.mesh.mesh  # [dp, tp] global ranks
    tpr = ctx.dims.tp_rank
    shard_group = replicate_group = None
    for t in range(tp):
        for n in range(nodes):
            ranks = [int(mesh[n * per_node_dp + i, t]) for i in range(per_node_dp)]
            g = dist.new_group(ranks)
            if t == tpr and n == dpr // per_node_dp:
                shard_group = g
        for i in range(per_node_dp):
            ranks = [int(mesh[n * per_node_dp + i, t]) for n in range(nodes)]
            g = dist.new_group(ranks)
            if t == tpr and i == dpr % per_node_dp:
                replicate_group = g
    return per_node_dp, dpr % per_node_dp, shard_group, replicate_group, nodes


def wrap_model_with_fsdp(model: nn.Module, ctx: Any, cfg: ParallelConfig,
                         transformer_layer_cls: Iterable[type[nn.Module]], *,
                         comm: Any = None) -> FullyShardedModel:
    """Shard ``model`` over the dp axis (API of ``src/parallelism/fsdp_utils.py:94``)."""
    from ..config import VALID_PREFETCH, VALID_SHARDING
    if cfg.sharding_strategy not in VALID_SHARDING:
        raise ValueError(f"Unknown sharding_strategy={cfg.sharding_strategy!r}; valid: "
                         f"{sorted(VALID_SHARDING)}.")
    if cfg.backward_prefetch not in VALID_PREFETCH:
        raise ValueError(f"Unknown backward_prefetch={cfg.backward_prefetch!r}; valid: "
                         f"{sorted(VALID_PREFETCH)}.")
    policy = build_mixed_precision(cfg)
    if policy.reduce_dtype != torch.float32:
        warnings.warn(f"reduce_dtype={cfg.reduce_dtype!r}: this engine accumulates and reduces gradients in "
                      "float32 regardless (more precise than the requested dtype).", stacklevel=2)
    return FullyShardedModel(model, ctx, cfg, transformer_layer_cls, comm=comm)


def apply_activation_checkpointing(model: nn.Module, transformer_layer_cls: Iterable[type[nn.Module]]) -> None:
    """Recompute each block's forward during backward (non-reentrant checkpoint).

    Same placement as ``src/parallelism/fsdp_utils.py:172-208``: it wraps the
    block's ``forward`` so hooks on the block still fire once per call.
    """
    from torch.utils.checkpoint import checkpoint
    classes = tuple(transformer_layer_cls)
    for m in model.modules():
        if isinstance(m, classes) and not getattr(m, "_ac_wrapped", False):
            inner = m.forward

            def fwd(*args, _inner=inner, **kw):
                if torch.is_grad_enabled():
                    return checkpoint(_inner, *args, use_reentrant=False, **kw)
                return _inner(*args, **kw)

            m.forward = fwd  # type: ignore[method-assign]
            m._ac_wrapped = True  # type: ignore[attr-defined]


def count_unsharded_parameters(model: nn.Module, ctx: Any) -> int:
    """Total parameter count across the dp shards (world all-reduce of local counts).

    For the sharded model the local count is the shard size minus this rank's
    share of padding, so the sum equals the unsharded model's count.
    """
    if isinstance(model, FullyShardedModel):
        local = 0
        for u in model.units:
            lo, hi = u.shard_range(model.shard_rank)
            for e in u.entries:
                a, b = max(lo, e.offset), min(hi, e.offset + e.numel)
                local += max(0, b - a)
        if model.dp_rank >= model.shard_world:
            local = 0  # NO_SHARD / HYBRID_SHARD replicas: count the first replica group only
        if model.tp_size > 1:
            # replicated entries exist on every TP rank: count them on tp_rank 0 only
            rep = 0
            for u in model.units:
                lo, hi = u.shard_range(model.shard_rank)
                for e in u.entries:
                    if e.tp_kind == "rep":
                        a, b = max(lo, e.offset), min(hi, e.offset + e.numel)
                        rep += max(0, b - a)
            if ctx.dims.tp_rank != 0 and model.dp_rank < model.shard_world:
                local -= rep
        t = torch.tensor([local], dtype=torch.long, device=ctx.device if ctx else "cpu")
    else:
        t = torch.tensor([sum(p.numel() for p in model.parameters())], dtype=torch.long,
                         device=ctx.device if ctx else "cpu")
    if dist.is_initialized():
        dist.all_reduce(t)
    return int(t.item())
