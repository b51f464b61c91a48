"""TP / 2-D numerics against a single-process oracle (gloo, fp32)."""

import copy

import pytest
import torch
import torch.distributed as dist

from build_your_own_distributed_training_b200.models.transformer import build_model
from build_your_own_distributed_training_b200.parallel.process_groups import build_process_context
from build_your_own_distributed_training_b200.parallel.tensor_parallel import apply_tensor_parallelism
from build_your_own_distributed_training_b200.training.trainer import build_engine
from tests._dist_utils import run_distributed
from tests.helpers import tiny_config


def _tp_logits_worker(rank, world):
    cfg = tiny_config()
    ctx = build_process_context(world, backend="gloo", verbose=False)
    torch.manual_seed(0)
    ref = build_model(cfg.model)
    tp_model = copy.deepcopy(ref)
    apply_tensor_parallelism(tp_model, ctx.tp_group)
    tok = torch.randint(0, 256, (3, 32), generator=torch.Generator().manual_seed(1))
    lab = torch.randint(0, 256, (3, 32), generator=torch.Generator().manual_seed(2))
    lr, ref_loss = ref(tok, labels=lab)
    lt, tp_loss = tp_model(tok, labels=lab)
    assert torch.allclose(lt, lr, atol=1e-4)
    ref_loss.backward()
    tp_loss.backward()
    # replicated params: identical grads; sharded params: this rank's slice
    for (n, p), (_, q) in zip(ref.named_parameters(), tp_model.named_parameters()):
        g = p.grad
        if q.shape != p.shape:
            dim = 0 if q.shape[0] != p.shape[0] else 1
            g = g.chunk(world, dim)[rank]
        assert torch.allclose(q.grad, g, atol=1e-5), n


def test_tp_logits_and_grads_match_single_device():
    run_distributed(_tp_logits_worker, 2)


def _2d_loss_worker(rank, world, sp, lp):
    """tp=2 x dp=2 loss and grad norm == one process on the union of both dp ranks' batches."""
    cfg = tiny_config(parallel__tp_size=2, parallel__sequence_parallel=sp, parallel__loss_parallel=lp)
    ctx = build_process_context(2, backend="gloo", verbose=False)
    cfg.validate(ctx.world_size, ctx.dims.dp_size, 2)
    eng = build_engine(cfg, ctx)
    torch.manual_seed(cfg.seed)
    ref = build_model(cfg.model)
    g = torch.Generator().manual_seed(11)
    toks = torch.randint(0, 256, (4, 33), generator=g)  # 2 sequences per dp rank
    mine = toks[ctx.dims.dp_rank * 2:(ctx.dims.dp_rank + 1) * 2]
    _, loss = eng(mine[:, :-1], labels=mine[:, 1:])
    loss.backward()
    lt = loss.detach().clone()
    dist.all_reduce(lt, group=ctx.dp_group)
    _, rl = ref(toks[:, :-1], labels=toks[:, 1:])
    rl.backward()
    assert abs(float(lt) / 2 - float(rl)) < 1e-5
    from build_your_own_distributed_training_b200.training.grad_utils import sharded_total_norm
    norm = float(sharded_total_norm(eng))
    ref_norm = float(torch.sqrt(sum(p.grad.pow(2).sum() for p in ref.parameters())))
    assert abs(norm - ref_norm) / ref_norm < 1e-4, (norm, ref_norm)


@pytest.mark.parametrize("sp,lp", [(False, False), (True, False), (False, True), (True, True)])
def test_2d_tp2_dp2_matches_union_oracle(sp, lp):
    run_distributed(_2d_loss_worker, 4, sp, lp)
