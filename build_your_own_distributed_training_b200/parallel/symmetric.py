"""NVLink transport: symmetric heaps and the collectives built on them.

Every rank of a group allocates one device buffer of the same size (a raw
``cudaMalloc``), exports it with a CUDA IPC handle, and maps every peer's
buffer, so each rank holds device pointers to all heaps of its group.  On one
NVSwitch node every GPU reaches every peer at full NVLink bandwidth, so the
collectives are single-step pulls run by this package's kernels
(``csrc/comm.cu``, ``csrc/gemm.cu``):

* :class:`PeerComm` - the ZeRO engine's transport over the dp group: the bf16
  parameter shards and the fp32 gradient buffers live in the heap; the
  all-gather pulls peers' shards, the reduce-scatter pulls this rank's slice
  of every peer's gradients and sums them in rank order with the 1/dp scale
  fused (deterministic, identical on every run);
* :class:`TPComm` - tensor parallelism: the row-parallel GEMM fused with its
  all-reduce (tiles are exchanged through the heap as the GEMM produces them,
  summed in rank order, residual added in the same epilogue), and the
  all-reduce / token all-gather / token reduce-scatter used elsewhere.

Synchronisation is by flags in the heaps (epochs, release/acquire at system
scope) with bounded waits: a peer that never arrives makes the kernel record
an error in the device error word and return, and the host raises
:class:`CollectiveTimeoutError` at the next step boundary.  ``torch.distributed``
is used only to exchange the IPC handles and for rare scalar reductions.
"""

from __future__ import annotations

import os
from typing import Any

import torch
import torch.distributed as dist

from ..ops._ext import native

TIMEOUT_S = float(os.environ.get("DTB_PEER_TIMEOUT_S", "10"))
_ALIGN = 256
_HEAPS: list["SymmetricHeap"] = []


class CollectiveTimeoutError(RuntimeError):
    """A peer-memory wait ran out: a peer died or stopped issuing collectives."""


def _align(n: int, a: int = _ALIGN) -> int:
    return -(-n // a) * a


class SymmetricHeap:
    """One same-sized device buffer per rank of ``group``, mapped into every rank."""

    def __init__(self, group: dist.ProcessGroup, nbytes: int, device: torch.device) -> None:
        self.group = group
        self.rank = dist.get_rank(group)
        self.size = dist.get_world_size(group)
        self.nbytes = _align(nbytes, 1 << 20)
        with torch.cuda.device(device):
            self.local = native().sym_malloc(self.nbytes)
        handle = native().ipc_handle(self.local).tolist()
        handles: list[Any] = [None] * self.size
        dist.all_gather_object(handles, handle, group=group)
        self.bases: list[int] = []
        self._opened: list[int] = []
        for r, h in enumerate(handles):
            if r == self.rank:
                self.bases.append(self.local.data_ptr())
            else:
                ptr = native().ipc_open(torch.tensor(h, dtype=torch.uint8))
                self.bases.append(ptr)
                self._opened.append(ptr)
        self._top = 0
        _HEAPS.append(self)

    def alloc(self, nbytes: int) -> int:
        off = self._top
        self._top = _align(off + nbytes)
        if self._top > self.nbytes:
            raise MemoryError(f"symmetric heap exhausted ({self._top} > {self.nbytes} bytes)")
        return off

    def view(self, off: int, numel: int, dtype: torch.dtype) -> torch.Tensor:
        nb = numel * torch.empty((), dtype=dtype).element_size()
        return self.local[off:off + nb].view(dtype)

    def offset_of(self, t: torch.Tensor) -> int:
        off = t.data_ptr() - self.local.data_ptr()
        if not 0 <= off < self.nbytes:
            raise ValueError("tensor is not inside this symmetric heap")
        return off

    def close(self) -> None:
        for p in self._opened:
            try:
                native().ipc_close(p)
            except RuntimeError:
                pass
        self._opened.clear()


def release_all() -> None:
    """Unmap every peer heap (call before the process group is destroyed)."""
    if torch.cuda.is_available() and _HEAPS:
        torch.cuda.synchronize()
    for h in _HEAPS:
        h.close()
    _HEAPS.clear()


def check_device_errors() -> None:
    """Raise if a kernel recorded a timeout or bad argument since the last check."""
    err = native().device_error()
    if err == 2:
        raise CollectiveTimeoutError(
            "a peer-memory wait timed out (a peer stopped participating); see DTB_PEER_TIMEOUT_S")
    if err:
        raise RuntimeError(f"device error word set: {err}")


class _Barrier:
    """Device barrier over a heap's group on one flag channel."""

    def __init__(self, heap: SymmetricHeap) -> None:
        self.heap = heap
        self.off = heap.alloc(128)
        self.epoch = 0

    def __call__(self) -> None:
        self.epoch += 1
        native().peer_barrier(self.heap.bases, self.off, self.heap.rank, self.epoch, TIMEOUT_S)


# ----------------------------------------------------------------------------- ZeRO (dp)
class PeerComm:
    """The sharding engine's transport over the dp group (see module docstring)."""

    name = "peer"

    def __init__(self, group: dist.ProcessGroup, device: torch.device) -> None:
        self.group = group
        self.size = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.rgroup, self.rsize = None, 1
        self.device = device
        self.heap: SymmetricHeap | None = None

    # the engine asks for all heap-resident buffers at once
    def alloc_many(self, specs: list[tuple[int, torch.dtype]]) -> list[torch.Tensor]:
        sizes = [_align(n * torch.empty((), dtype=d).element_size()) for n, d in specs]
        self.heap = SymmetricHeap(self.group, sum(sizes) + 64 * 1024, self.device)
        self._step_barrier = _Barrier(self.heap)
        self._rs_barrier = _Barrier(self.heap)
        out = []
        for (n, d), nb in zip(specs, sizes):
            out.append(self.heap.view(self.heap.alloc(nb), n, d))
        return out

    def barrier(self) -> None:
        if self.heap is not None:
            self._step_barrier()

    # parameter all-gathers on the copy engines (no SM work beside the GEMMs) unless
    # DTB_AG_COPY_ENGINE=0 selects the SM pull kernel
    ag_copy_engine = os.environ.get("DTB_AG_COPY_ENGINE", "1") != "0"

    def all_gather(self, out_full: torch.Tensor, shard: torch.Tensor) -> None:
        assert self.heap is not None
        nbytes = shard.numel() * shard.element_size()
        if self.ag_copy_engine:
            native().peer_all_gather_ce(self.heap.bases, self.heap.offset_of(shard), nbytes, out_full)
        else:
            native().peer_all_gather(self.heap.bases, self.heap.offset_of(shard), nbytes, out_full)

    # the reduce-scatter also leaves per-block partial sums of squares of its result
    norm_partials = True

    @staticmethod
    def norm_partial_blocks(shard_numel: int) -> int:
        return int(native().reduce_scatter_blocks(shard_numel))

    def reduce_scatter_mean(self, out_shard: torch.Tensor, full: torch.Tensor, world: int,
                            part: torch.Tensor | None = None, split: int = 0, rep_w: float = 1.0) -> None:
        """``out_shard = mean over ranks of this rank's slice of full``; with ``part``, also
        ``part[b] = sum over block b of w_i * out_i^2`` (``w_i = 1`` below ``split``, else ``rep_w``)."""
        assert self.heap is not None
        self._rs_barrier()  # every rank finished accumulating this unit's gradients
        native().peer_reduce_scatter(self.heap.bases, self.heap.offset_of(full), self.rank, 1.0 / world,
                                     out_shard, part, split, rep_w)

    def all_reduce_sum(self, t: torch.Tensor, group: dist.ProcessGroup | None) -> None:
        dist.all_reduce(t, group=group)


class PeerReplicaComm(PeerComm):
    """NO_SHARD over the NVLink transport: every rank keeps whole units, and the
    gradient all-reduce runs in place in the heap-resident gradient buffers as a
    reduce-scatter (rank r sums slice r of every rank's buffer into its own, rank
    order, 1/dp fused) followed by a copy-engine all-gather of the reduced slices.
    Peers finish reading a rank's slice before that rank writes gradients again:
    the step barrier after the optimizer step orders it."""

    name = "peer-replica"
    norm_partials = False

    def __init__(self, group: dist.ProcessGroup, device: torch.device) -> None:
        super().__init__(group, device)
        # the engine's view: one shard holds the whole unit, replicated on `size` ranks
        self.dp_size, self.dp_rank = self.size, self.rank
        self.size, self.rank = 1, 0
        self.rgroup, self.rsize = group, self.dp_size

    def alloc_many(self, specs: list[tuple[int, torch.dtype]]) -> list[torch.Tensor]:
        out = super().alloc_many(specs)
        self._ag_barrier = _Barrier(self.heap)
        return out

    def all_gather(self, out_full: torch.Tensor, shard: torch.Tensor) -> None:
        if out_full.data_ptr() != shard.data_ptr():
            out_full.copy_(shard)

    def reduce_scatter_mean(self, out_shard: torch.Tensor, full: torch.Tensor, world: int,
                            part: torch.Tensor | None = None, split: int = 0, rep_w: float = 1.0) -> None:
        assert self.heap is not None and out_shard.data_ptr() == full.data_ptr()
        n, d = full.numel(), self.dp_size
        if n % (4 * d) != 0:  # slices must stay 16-byte aligned: plain all-reduce for this unit
            dist.all_reduce(full, group=self.group)
            full.div_(world)
            return
        per = n // d
        off = self.heap.offset_of(full)
        self._rs_barrier()  # every rank's gradients of this unit are complete
        # slice r of every rank, summed into this rank's own slice r (each element is read
        # by the thread that then overwrites it; peers read only their own slices)
        mine = full[self.dp_rank * per:(self.dp_rank + 1) * per]
        native().peer_reduce_scatter(self.heap.bases, off, self.dp_rank, 1.0 / world, mine, None, 0, 1.0)
        self._ag_barrier()  # every slice reduced
        native().peer_all_gather_ce(self.heap.bases, off, per * 4, full, per * 4, self.dp_rank)


# ----------------------------------------------------------------------------- TP
class _RowParallelAR(torch.autograd.Function):
    """``y = all_reduce(x @ W^T) + residual`` with the all-reduce inside the GEMM."""

    @staticmethod
    def forward(ctx, x2, weight, residual, main_grad, comm):  # type: ignore[override]
        out = comm.gemm_all_reduce(x2, weight, residual)
        ctx.save_for_backward(x2, weight)
        ctx.main_grad = main_grad
        ctx.has_res = residual is not None
        return out

    @staticmethod
    def backward(ctx, dy):  # type: ignore[override]
        from ..ops import gemm
        x2, w = ctx.saved_tensors
        dy = dy.contiguous()
        dx = gemm.mm_nn(dy, w)  # the input is TP-sharded: no reduction needed
        if ctx.main_grad is not None:
            gemm.mm_tn_into_grad(dy, x2, ctx.main_grad, w.shape)
            dw = None
        else:
            dw = gemm.mm_tn(dy, x2).to(w.dtype) if w.requires_grad else None
        return dx, dw, (dy if ctx.has_res else None), None, None


class _RowParallelRS(torch.autograd.Function):
    """Sequence parallel: ``y = reduce_scatter_rows(x @ W^T) + residual`` in one kernel.

    Backward: the output gradient (this rank's rows) is all-gathered by pull,
    then the input and weight gradients are plain GEMMs.
    """

    @staticmethod
    def forward(ctx, x2, weight, residual, main_grad, comm):  # type: ignore[override]
        out = comm.gemm_reduce_scatter(x2, weight, residual)
        ctx.save_for_backward(x2, weight)
        ctx.main_grad = main_grad
        ctx.has_res = residual is not None
        ctx.comm = comm
        return out

    @staticmethod
    def backward(ctx, dy):  # type: ignore[override]
        from ..ops import gemm
        x2, w = ctx.saved_tensors
        dy_full = ctx.comm.all_gather_rows(dy.contiguous())
        dx = gemm.mm_nn(dy_full, w)
        if ctx.main_grad is not None:
            gemm.mm_tn_into_grad(dy_full, x2, ctx.main_grad, w.shape)
            dw = None
        else:
            dw = gemm.mm_tn(dy_full, x2).to(w.dtype) if w.requires_grad else None
        return dx, dw, (dy if ctx.has_res else None), None, None


class TPComm:
    """Tensor-parallel collectives over NVLink for one TP group."""

    def __init__(self, group: dist.ProcessGroup, device: torch.device, max_tokens: int, width: int) -> None:
        self.group = group
        self.size = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.max_tokens, self.width = max_tokens, width
        self.max_elems = max_tokens * width
        # one flag per (128-row slab, column block, quadrant, rank), then one "done" flag per
        # (slab, block, quadrant) for the two-shot all-reduce; +1 slab row covers 256-row
        # CTA-pair tiles that overhang max_tokens
        tiles = (-(-max_tokens // 128) + 1) * (-(-width // 128))
        self.flag_bytes = _align(tiles * 4 * (self.size + 1) * 4)
        # two-shot (owner sums, others copy) once one-shot ingress, (tp-1) payloads per rank,
        # exceeds two-shot's 2(tp-1)/tp; DTB_TP_TWO_SHOT=0/1 overrides
        env = os.environ.get("DTB_TP_TWO_SHOT")
        self.two_shot = (env == "1") if env in ("0", "1") else self.size >= 4
        # the layers use the fused all-reduces (GEMM + all-reduce, dgrad + all-reduce, standalone)
        # up to tp = 4; at tp = 8 GEMM + NCCL all-reduce measured faster in every 7B shape
        # (0.31-0.37 ms against 0.39-0.48 ms two-shot, tests/performance/bench_fused_comm.py),
        # so they take that path there.  DTB_TP_FUSED_AR_MAX moves the limit.
        self.fused_ar = self.size <= int(os.environ.get("DTB_TP_FUSED_AR_MAX", "4"))
        slot = _align(self.max_elems * 2)
        self.heap = SymmetricHeap(group, 2 * slot + self.flag_bytes + 64 * 1024, device)
        self.slots = [self.heap.alloc(slot), self.heap.alloc(slot)]
        self.flag_off = self.heap.alloc(self.flag_bytes)
        self.ag_flag_off = self.heap.alloc(256)  # per-rank "rows staged" flags of the fused all-gather GEMM
        self.barrier = _Barrier(self.heap)
        self.calls = 0

    def _slot(self) -> int:
        self.calls += 1
        return self.slots[self.calls % 2]

    def _staging(self, off: int, shape: tuple[int, ...]) -> torch.Tensor:
        n = 1
        for s in shape:
            n *= s
        if n > self.max_elems:
            raise ValueError(f"TP staging holds {self.max_elems} elements, {n} requested")
        return self.heap.view(off, n, torch.bfloat16).view(shape)

    # fused GEMM -> all-reduce (+ residual)
    def gemm_all_reduce(self, x2: torch.Tensor, w: torch.Tensor, residual: torch.Tensor | None) -> torch.Tensor:
        M, N = x2.shape[0], w.shape[0]
        if M > self.max_tokens or N > self.width:
            raise ValueError(f"row-parallel output [{M}, {N}] exceeds the TP staging area "
                             f"[{self.max_tokens}, {self.width}]")
        out = torch.empty(M, N, device=x2.device, dtype=torch.bfloat16)
        off = self._slot()
        native().gemm_peer_ar(x2, w, out, False, residual, None, self.heap.bases, self.rank, off, self.flag_off,
                              self.calls, TIMEOUT_S, self.two_shot)
        return out

    # fused input-gradient GEMM -> all-reduce of a column-parallel layer: dy @ W, summed over TP
    def gemm_all_reduce_dgrad(self, dy: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        M, K = dy.shape[0], w.shape[1]
        if M > self.max_tokens or K > self.width:
            raise ValueError(f"input gradient [{M}, {K}] exceeds the TP staging area "
                             f"[{self.max_tokens}, {self.width}]")
        out = torch.empty(M, K, device=dy.device, dtype=torch.bfloat16)
        off = self._slot()
        native().gemm_peer_ar(dy.contiguous(), w, out, True, None, None, self.heap.bases, self.rank, off,
                              self.flag_off, self.calls, TIMEOUT_S, self.two_shot)
        return out

    # fused GEMM -> reduce-scatter of rows (+ residual in the scattered layout)
    def gemm_reduce_scatter(self, x2: torch.Tensor, w: torch.Tensor, residual: torch.Tensor | None) -> torch.Tensor:
        M, N = x2.shape[0], w.shape[0]
        if M > self.max_tokens or N > self.width:
            raise ValueError(f"row-parallel output [{M}, {N}] exceeds the TP staging area "
                             f"[{self.max_tokens}, {self.width}]")
        rows = M // self.size
        out = torch.empty(rows, N, device=x2.device, dtype=torch.bfloat16)
        off = self._slot()
        native().gemm_peer_rs(x2, w, out, False, residual, self.heap.bases, self.rank, off, self.flag_off,
                              self.calls, TIMEOUT_S, self.rank * rows, rows)
        return out

    def row_parallel_linear(self, x2, weight, residual, main_grad):
        if self._sequence_parallel:
            rows = x2.shape[0] // self.size
            if x2.shape[0] % self.size == 0 and rows % 128 == 0:
                return _RowParallelRS.apply(x2.contiguous(), weight, residual, main_grad, self)
            from ..ops.linear import linear
            y = linear(x2, weight, main_grad=main_grad)
            y = _SeqReduceScatterPeer.apply(y, self)
            return y + residual if residual is not None else y
        return _RowParallelAR.apply(x2.contiguous(), weight, residual, main_grad, self)

    _sequence_parallel = False

    # ---- sequence parallelism: column-parallel GEMMs with the token all-gather fused in
    # front (forward) and the input gradient fused with its reduce-scatter (backward)
    def sp_fusable(self, x_local: torch.Tensor) -> bool:
        R, K = x_local.shape
        return (R % 256 == 0 and R * self.size <= self.max_tokens and K <= self.width and K % 8 == 0
                and x_local.dtype == torch.bfloat16)

    def _stage_rows(self, x_local: torch.Tensor) -> int:
        off = self._slot()
        self._staging(off, tuple(x_local.shape)).copy_(x_local)
        native().peer_signal(self.heap.bases, self.ag_flag_off, self.rank, self.calls)
        return off

    def gather_gemm(self, x_local: torch.Tensor, w: torch.Tensor, epi: int, *, cos=None, sin=None, p0: int = 0,
                    p1: int = 0, ffn: int = 0) -> tuple[Any, torch.Tensor]:
        """``(y, x_gathered)``: ``y = all_gather_rows(x_local) @ w^T`` with the given epilogue
        (0 store, 4 RoPE, 5 SwiGLU: ``y = (act, [g|u])``), the gather inside the GEMM."""
        x_local = x_local.contiguous()
        R, K = x_local.shape
        M = R * self.size
        off = self._stage_rows(x_local)
        xg = torch.empty(M, K, device=x_local.device, dtype=x_local.dtype)
        if epi == 5:
            act = torch.empty(M, ffn, device=x_local.device, dtype=x_local.dtype)
            gu = torch.empty(M, 2 * ffn, device=x_local.device, dtype=x_local.dtype)
            native().gemm_ag(xg, x_local, w, act, 5, None, None, gu, ffn, 0, self.heap.bases, self.rank, off,
                             self.ag_flag_off, self.calls, TIMEOUT_S)
            return (act, gu), xg
        out = torch.empty(M, w.shape[0], device=x_local.device, dtype=x_local.dtype)
        native().gemm_ag(xg, x_local, w, out, epi, cos, sin, None, p0, p1, self.heap.bases, self.rank, off,
                         self.ag_flag_off, self.calls, TIMEOUT_S)
        return out, xg

    def dgrad_reduce_scatter(self, dy: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        """This rank's rows of ``sum over the group of dy @ w`` (``w``: ``[N, K]``) in one kernel."""
        M, K = dy.shape[0], w.shape[1]
        if M > self.max_tokens or K > self.width:
            raise ValueError(f"input gradient [{M}, {K}] exceeds the TP staging area "
                             f"[{self.max_tokens}, {self.width}]")
        rows = M // self.size
        out = torch.empty(rows, K, device=dy.device, dtype=torch.bfloat16)
        off = self._slot()
        native().gemm_peer_rs(dy.contiguous(), w, out, True, None, self.heap.bases, self.rank, off, self.flag_off,
                              self.calls, TIMEOUT_S, self.rank * rows, rows)
        return out

    # per-row records exchanged by the fused vocabulary-parallel cross-entropy
    def exchange_rows(self, rows: int, row_bytes: int) -> tuple[int, torch.Tensor]:
        """A staging slot for ``rows`` records of ``row_bytes`` (a multiple of 4): (offset, fp32 view)."""
        off = self._slot()
        if rows * row_bytes > self.max_elems * 2:
            raise ValueError(f"TP staging holds {self.max_elems * 2} bytes, {rows * row_bytes} requested")
        return off, self.heap.view(off, rows * row_bytes // 4, torch.float32)

    def exchange_publish(self, off: int, rows: torch.Tensor) -> tuple[list[int], int]:
        """After every rank filled its slot: (heap base of every rank, offset) to read them at."""
        self.barrier()
        return self.heap.bases, off

    # standalone collectives on bf16 activations
    def all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        x = x.contiguous()
        if self.two_shot and x.dim() >= 2 and x.shape[0] % self.size == 0 \
                and (x.numel() // x.shape[0]) % 8 == 0:
            # two-shot: each rank sums its row block from every peer, then every rank
            # pulls every block (2(tp-1)/tp payloads in, against tp-1 one-shot)
            return self.all_gather_rows(self.reduce_scatter_rows(x))
        off = self._slot()
        self._staging(off, tuple(x.shape)).copy_(x)
        self.barrier()
        out = torch.empty_like(x)
        native().peer_all_reduce_bf16(self.heap.bases, off, None, out)
        return out

    def all_gather_rows(self, x: torch.Tensor) -> torch.Tensor:
        x = x.contiguous()
        off = self._slot()
        self._staging(off, tuple(x.shape)).copy_(x)
        self.barrier()
        out = torch.empty((x.shape[0] * self.size,) + tuple(x.shape[1:]), device=x.device, dtype=x.dtype)
        native().peer_all_gather(self.heap.bases, off, x.numel() * x.element_size(), out)
        return out

    def reduce_scatter_rows(self, x: torch.Tensor) -> torch.Tensor:
        x = x.contiguous()
        rows = x.shape[0] // self.size
        cols = x.numel() // x.shape[0]
        off = self._slot()
        self._staging(off, tuple(x.shape)).copy_(x)
        self.barrier()
        out = torch.empty((rows,) + tuple(x.shape[1:]), device=x.device, dtype=x.dtype)
        native().peer_reduce_rows_bf16(self.heap.bases, off, self.rank * rows, cols, out)
        return out


class _SeqReduceScatterPeer(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, comm):  # type: ignore[override]
        ctx.comm = comm
        return comm.reduce_scatter_rows(x)

    @staticmethod
    def backward(ctx, g):  # type: ignore[override]
        return ctx.comm.all_gather_rows(g.contiguous()), None


def build_comms(ctx: Any, config: Any) -> tuple[TPComm | None, PeerComm | None]:
    """Transports for this rank: ``(tp_comm, dp_comm)`` (``None`` for size-1 groups)."""
    dev = ctx.device
    tp = dp = None
    if ctx.dims.tp_size > 1:
        tokens = config.data.micro_batch_size * config.data.seq_len
        tp = TPComm(ctx.tp_group, dev, tokens, config.model.d_model)
        tp._sequence_parallel = bool(config.parallel.sequence_parallel)
    strategy = config.parallel.sharding_strategy
    dp_size = ctx.dims.dp_size
    # HYBRID_SHARD shards inside a node: on one node that is the whole dp group
    one_node = max(1, ctx.env.local_world_size // ctx.dims.tp_size) >= dp_size
    if 1 < dp_size <= 8:
        if strategy in ("FULL_SHARD", "SHARD_GRAD_OP") or (strategy == "HYBRID_SHARD" and one_node):
            dp = PeerComm(ctx.dp_group, dev)
        elif strategy == "NO_SHARD" and one_node:
            dp = PeerReplicaComm(ctx.dp_group, dev)
    return tp, dp
