"""The ZeRO-3 engine on gloo ranks: layout, sharding invariants, gradients, policies."""

import pytest
import torch
import torch.distributed as dist

from build_your_own_distributed_training_b200.models.transformer import TransformerBlock, build_model
from build_your_own_distributed_training_b200.parallel.fsdp import count_unsharded_parameters
from build_your_own_distributed_training_b200.parallel.process_groups import build_process_context
from build_your_own_distributed_training_b200.training.trainer import build_engine
from tests._dist_utils import run_distributed
from tests.helpers import tiny_config


def _layout_worker(rank, world, strategy):
    cfg = tiny_config(parallel__sharding_strategy=strategy)
    ctx = build_process_context(1, backend="gloo", verbose=False)
    torch.manual_seed(cfg.seed)
    full = build_model(cfg.model)
    eng = build_engine(cfg, ctx)
    # every unit: [wq; wk; wv] and [gate; up] adjacent, matrices before vectors
    blk = eng.units[0]
    names = [e.fqn.split(".", 2)[-1] for e in blk.entries]
    assert names[:7] == ["attention.wq.weight", "attention.wk.weight", "attention.wv.weight",
                         "attention.wo.weight", "mlp.gate_proj.weight", "mlp.up_proj.weight",
                         "mlp.down_proj.weight"]
    assert blk.decay_end == blk.entries[-2].offset  # norms after the matrices
    # sharding invariant: the sum of local pieces is the model size (tied weight counted once)
    n = count_unsharded_parameters(eng, ctx)
    assert n == sum(p.numel() for p in full.parameters())
    # gathered params equal the original full weights
    for u in eng.units:
        eng._ensure(u.index) if u.index < len(eng.blocks) else None
        for e in u.entries:
            want = dict(full.named_parameters())[e.fqn]
            assert torch.equal(e.param.detach(), want.detach()), e.fqn
    _, loss = eng(torch.randint(0, 256, (2, 16)), labels=torch.randint(0, 256, (2, 16)))
    loss.backward()
    assert torch.isfinite(loss)
    for u in eng.units:
        assert torch.isfinite(u.grad_shard).all()


@pytest.mark.parametrize("strategy", ["FULL_SHARD", "SHARD_GRAD_OP", "NO_SHARD", "HYBRID_SHARD"])
def test_engine_layout_and_invariants(strategy):
    run_distributed(_layout_worker, 2, strategy)


def _grad_equivalence_worker(rank, world, strategy):
    """Sharded grads (mean over dp) equal the single-process grad of the global batch."""
    cfg = tiny_config(parallel__sharding_strategy=strategy)
    ctx = build_process_context(1, backend="gloo", verbose=False)
    eng = build_engine(cfg, ctx)
    torch.manual_seed(cfg.seed)
    ref = build_model(cfg.model)
    g = torch.Generator().manual_seed(7)
    toks = torch.randint(0, 256, (world * 2, 17), generator=g)
    mine = toks[rank * 2:(rank + 1) * 2]
    _, loss = eng(mine[:, :-1], labels=mine[:, 1:])
    loss.backward()
    _, rl = ref(toks[:, :-1], labels=toks[:, 1:])
    rl.backward()
    named = dict(ref.named_parameters())
    for u in eng.units:
        lo, hi = u.shard_range(eng.shard_rank)
        flat = torch.zeros(u.numel)
        for e in u.entries:
            flat[e.offset:e.offset + e.numel] = named[e.fqn].grad.reshape(-1)
        assert torch.allclose(u.grad_shard, flat[lo:hi], atol=1e-6, rtol=1e-4)


@pytest.mark.parametrize("strategy", ["FULL_SHARD", "NO_SHARD"])
def test_dp_grads_equal_global_batch(strategy):
    run_distributed(_grad_equivalence_worker, 2, strategy)


def _no_sync_worker(rank, world):
    cfg = tiny_config()
    ctx = build_process_context(1, backend="gloo", verbose=False)
    eng = build_engine(cfg, ctx)
    g = torch.Generator().manual_seed(rank)
    a, b = torch.randint(0, 256, (2, 17), generator=g), torch.randint(0, 256, (2, 17), generator=g)
    with eng.no_sync():
        _, l1 = eng(a[:, :-1], labels=a[:, 1:])
        (l1 / 2).backward()
    shard_before = [u.grad_shard.clone() for u in eng.units]
    _, l2 = eng(b[:, :-1], labels=b[:, 1:])
    (l2 / 2).backward()
    acc = [u.grad_shard.clone() for u in eng.units]
    # the no_sync micro-step did not reduce anything
    assert all(torch.equal(s, torch.zeros_like(s)) for s in shard_before)
    eng.zero_grad_buffers()
    ab = torch.cat([a, b])
    _, lf = eng(ab[:, :-1], labels=ab[:, 1:])
    lf.backward()
    for x, y in zip(acc, [u.grad_shard for u in eng.units]):
        assert torch.allclose(x, y, atol=1e-6, rtol=1e-4)


def test_no_sync_accumulation_equals_full_batch():
    run_distributed(_no_sync_worker, 2)


def test_mixed_precision_policy():
    from build_your_own_distributed_training_b200.config import ParallelConfig
    from build_your_own_distributed_training_b200.utils.dtype import (autocast_dtype, build_mixed_precision,
                                                                     resolve_dtype)
    pol = build_mixed_precision(ParallelConfig())
    assert (pol.param_dtype, pol.reduce_dtype, pol.master_dtype) == (torch.bfloat16, torch.float32, torch.float32)
    assert autocast_dtype(ParallelConfig()) == torch.bfloat16
    assert resolve_dtype("BF16") == torch.bfloat16 and resolve_dtype("half") == torch.float16
    with pytest.raises(ValueError):
        resolve_dtype("fp8")


def _bf16_engine_worker(rank, world):
    cfg = tiny_config(parallel__param_dtype="bfloat16")
    ctx = build_process_context(1, backend="gloo", verbose=False)
    eng = build_engine(cfg, ctx)
    for u in eng.units:
        assert u.master.dtype == torch.float32 and u.param_shard.dtype == torch.bfloat16
        assert u.grad.dtype == torch.float32
        for e in u.entries:
            assert e.param.dtype == torch.bfloat16 and e.param.main_grad.dtype == torch.float32
    dist.barrier()


def test_bf16_params_fp32_master_and_grads():
    run_distributed(_bf16_engine_worker, 2)


def _memory_bound_worker(rank, world, limit):
    cfg = tiny_config(parallel__sharding_strategy="FULL_SHARD", parallel__limit_all_gathers=limit,
                      model__n_layers=4)
    ctx = build_process_context(1, backend="gloo", verbose=False)
    eng = build_engine(cfg, ctx)
    blocks = eng.units[:-1]
    slots = {s.data_ptr() for s in eng._slots}
    assert len(slots) == (2 if limit else 3)
    # every block's gathered parameters live in one of the rotating slots
    assert {u.gathered.data_ptr() for u in blocks} == slots
    _, loss = eng(torch.randint(0, 256, (2, 16)), labels=torch.randint(0, 256, (2, 16)))
    loss.backward()
    assert torch.isfinite(loss)


@pytest.mark.parametrize("limit", [True, False])
def test_gathered_blocks_are_bounded(limit):
    """At most two (limit_all_gathers) or three gathered blocks exist at any time."""
    run_distributed(_memory_bound_worker, 2, limit)


def _prefetch_order_worker(rank, world, mode, out):
    cfg = tiny_config(parallel__sharding_strategy="FULL_SHARD", parallel__backward_prefetch=mode,
                      model__n_layers=3)
    ctx = build_process_context(1, backend="gloo", verbose=False)
    eng = build_engine(cfg, ctx)
    events = []
    orig_post = eng._post_backward
    eng._prefetch = lambda bi: events.append(("prefetch", bi))

    def post(bi):
        events.append(("post", bi))
        orig_post(bi)
    eng._post_backward = post
    _, loss = eng(torch.randint(0, 256, (2, 16)), labels=torch.randint(0, 256, (2, 16)))
    events.clear()  # keep the backward only
    loss.backward()
    out.extend(events)


@pytest.mark.parametrize("mode", ["BACKWARD_PRE", "BACKWARD_POST"])
def test_backward_prefetch_order(single_process_pg, mode):
    """BACKWARD_PRE gathers block i-1 when block i's backward starts; BACKWARD_POST once it ends."""
    events = []
    _prefetch_order_worker(0, 1, mode, events)
    i_pre = events.index(("prefetch", 1))
    i_post = events.index(("post", 2))
    assert (i_pre < i_post) if mode == "BACKWARD_PRE" else (i_pre > i_post), events


def _norm_terms_worker(rank, world, tp):
    """The per-unit sums of squares taken right after each unit's reduction give the same
    norm bits as a pass over the gradient shards after the backward, and are not used once a
    backward that reduced nothing (no_sync) has changed the gradients."""
    cfg = tiny_config(parallel__tp_size=tp)
    ctx = build_process_context(tp, backend="gloo", verbose=False)
    eng = build_engine(cfg, ctx)
    g = torch.Generator().manual_seed(3 + rank // tp)
    toks = torch.randint(0, 256, (2, 17), generator=g)
    _, loss = eng(toks[:, :-1], labels=toks[:, 1:])
    loss.backward()
    eng.wait_reduce()
    assert eng._unit_ss is not None and all(eng._ss_fresh)
    early = eng.grad_norm_sq_local().clone()
    eng._ss_fresh = [False] * len(eng.units)
    late = eng.grad_norm_sq_local()
    assert torch.equal(early, late) and float(late) > 0
    eng._ss_fresh = [True] * len(eng.units)
    with eng.no_sync():
        _, l2 = eng(toks[:, :-1], labels=toks[:, 1:])
        l2.backward()
    assert not any(eng._ss_fresh)


@pytest.mark.parametrize("tp", [1, 2])
def test_norm_terms_after_each_reduction_match_a_pass(tp):
    run_distributed(_norm_terms_worker, 2, tp)
