"""Optimizer steps against torch.optim and the written-out LAMB formula.

The sharded AdamW update (CPU path of the fused kernel) must equal
``torch.optim.AdamW`` step for step; the clip state ``[coef, finite]`` scales
the gradient or skips the step; LAMB matches the layer-wise trust-ratio
formula; and sharded LAMB over two ranks equals the one-rank result, which
checks the all-reduced per-tensor norms.
"""
import torch

from build_your_own_distributed_training_b200.parallel.process_groups import build_process_context
from build_your_own_distributed_training_b200.parallel.state_dict import get_model_state_dict
from build_your_own_distributed_training_b200.training.loop import train_step
from build_your_own_distributed_training_b200.training.optimizer import LAMB, _adamw_ref
from build_your_own_distributed_training_b200.training.trainer import Trainer
from tests._dist_utils import run_distributed
from tests.helpers import tiny_config

LR, B1, B2, EPS, WD = 1e-2, 0.9, 0.95, 1e-8, 0.1


def _grads(n, steps, seed=0):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(n, generator=g) for _ in range(steps)]


def test_adamw_update_equals_torch_adamw():
    p0 = torch.randn(1000, generator=torch.Generator().manual_seed(1))
    ref = p0.clone().requires_grad_()
    opt = torch.optim.AdamW([ref], lr=LR, betas=(B1, B2), eps=EPS, weight_decay=WD, foreach=False)
    p, m, v = p0.clone(), torch.zeros(1000), torch.zeros(1000)
    out = torch.empty(1000, dtype=torch.bfloat16)
    for t, g in enumerate(_grads(1000, 5), start=1):
        ref.grad = g.clone()
        opt.step()
        _adamw_ref(p, g, m, v, out, None, LR, B1, B2, EPS, WD, t)
        torch.testing.assert_close(p, ref.detach(), rtol=1e-6, atol=1e-7)
    assert torch.equal(out, p.to(torch.bfloat16))


def test_adamw_clip_state_scales_or_skips():
    p0 = torch.randn(64)
    g = torch.randn(64)
    a, m1, v1 = p0.clone(), torch.zeros(64), torch.zeros(64)
    b, m2, v2 = p0.clone(), torch.zeros(64), torch.zeros(64)
    out = torch.empty(64, dtype=torch.bfloat16)
    _adamw_ref(a, g, m1, v1, out, torch.tensor([0.25, 1.0]), LR, B1, B2, EPS, WD, 1)
    _adamw_ref(b, g * 0.25, m2, v2, out, None, LR, B1, B2, EPS, WD, 1)
    assert torch.equal(a, b) and torch.equal(m1, m2) and torch.equal(v1, v2)
    c, m3, v3 = p0.clone(), torch.zeros(64), torch.zeros(64)
    _adamw_ref(c, g, m3, v3, out, torch.tensor([1.0, 0.0]), LR, B1, B2, EPS, WD, 1)
    assert torch.equal(c, p0) and not m3.any() and not v3.any()


def test_lamb_matches_formula():
    torch.manual_seed(0)
    w = torch.randn(8, 16)
    b = torch.randn(16)
    pw, pb = w.clone().requires_grad_(), b.clone().requires_grad_()
    opt = LAMB([{"params": [pw], "weight_decay": WD}, {"params": [pb], "weight_decay": 0.0}],
               lr=LR, betas=(B1, B2), eps=1e-6)
    state = {"w": [w.clone(), torch.zeros_like(w), torch.zeros_like(w), WD],
             "b": [b.clone(), torch.zeros_like(b), torch.zeros_like(b), 0.0]}
    for t in range(1, 4):
        gw, gb = torch.randn(8, 16), torch.randn(16)
        pw.grad, pb.grad = gw.clone(), gb.clone()
        opt.step()
        for key, g in (("w", gw), ("b", gb)):
            x, m, v, wd = state[key]
            m.mul_(B1).add_((1 - B1) * g)
            v.mul_(B2).add_((1 - B2) * g * g)
            r = (m / (1 - B1 ** t)) / ((v / (1 - B2 ** t)).sqrt() + 1e-6) + wd * x
            trust = x.norm() / r.norm()
            x.sub_(LR * trust * r)
    torch.testing.assert_close(pw.detach(), state["w"][0], rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(pb.detach(), state["b"][0], rtol=1e-5, atol=1e-6)


def _lamb_run(rank, world, out_path):
    ctx = build_process_context(1, backend="gloo", verbose=False)
    cfg = tiny_config(None, optimizer__name="lamb", data__global_batch_size=16, data__micro_batch_size=8 // world)
    t = Trainer(cfg, ctx=ctx, gpu_type="cpu")
    for _ in range(3):
        w, _ = t._next_window()
        train_step(t.model, w, t.optimizer, t.scheduler, ctx, cfg, gpu_type="cpu")
    sd = get_model_state_dict(t.model, full=True)
    if rank == 0:
        torch.save(sd, out_path)


def test_sharded_lamb_is_invariant_to_the_shard_count(tmp_path):
    one, two = str(tmp_path / "w1.pt"), str(tmp_path / "w2.pt")
    run_distributed(_lamb_run, 1, one)
    run_distributed(_lamb_run, 2, two)
    a, b = torch.load(one), torch.load(two)
    assert a.keys() == b.keys()
    for k in a:
        torch.testing.assert_close(a[k], b[k], rtol=1e-4, atol=1e-5, msg=k)
