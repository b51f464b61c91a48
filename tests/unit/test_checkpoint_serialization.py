"""Round trips of the checkpoint format, and loading under weights_only=True."""

import os

import torch

from build_your_own_distributed_training_b200.checkpointing.checkpoint import load_checkpoint, save_checkpoint
from build_your_own_distributed_training_b200.parallel.process_groups import build_process_context
from build_your_own_distributed_training_b200.training.loop import train_step
from build_your_own_distributed_training_b200.training.trainer import Trainer
from tests.helpers import tiny_config


def test_save_load_roundtrip_and_weights_only(tmp_path, single_process_pg):
    cfg = tiny_config(str(tmp_path), run_id="rt")
    ctx = build_process_context(1, backend="gloo", verbose=False)
    tr = Trainer(cfg, ctx=ctx, gpu_type="cpu")
    for _ in range(3):
        w, _ = tr._next_window()
        train_step(tr.model, w, tr.optimizer, tr.scheduler, ctx, cfg, gpu_type="cpu")
    path = save_checkpoint(tr.model, tr.optimizer, tr.scheduler, 3, cfg, ctx)
    for f in ("model.pt", "optim.pt", "rng.pt"):
        torch.load(os.path.join(path, "rank_0", f), weights_only=True)  # no pickle needed
    sd = torch.load(os.path.join(path, "rank_0", "model.pt"), weights_only=True)
    assert "layers.0.attention.wq.weight" in sd and "lm_head.weight" in sd and "tok_embeddings.weight" in sd
    osd = torch.load(os.path.join(path, "rank_0", "optim.pt"), weights_only=True)
    assert set(osd["state"]["layers.1.mlp.down_proj.weight"]) == {"step", "exp_avg", "exp_avg_sq"}
    assert open(os.path.join(path, "_SUCCESS")).read() == "3"
    tr2 = Trainer(tiny_config(str(tmp_path), run_id="rt"), ctx=ctx, gpu_type="cpu")
    step = load_checkpoint(tr2.model, tr2.optimizer, tr2.scheduler, path, ctx)
    assert step == 3
    for a, b in zip(tr.model.units, tr2.model.units):
        assert torch.equal(a.master, b.master)
        sa, sb = tr.optimizer.state[a.master], tr2.optimizer.state[b.master]
        assert torch.equal(sa["exp_avg"], sb["exp_avg"]) and torch.equal(sa["exp_avg_sq"], sb["exp_avg_sq"])
    tok = torch.randint(0, 256, (2, 16))
    assert torch.equal(tr.model(tok, labels=tok)[1], tr2.model(tok, labels=tok)[1])


def test_plain_module_state_dict_roundtrip(tmp_path):
    from build_your_own_distributed_training_b200.models.transformer import build_model
    from build_your_own_distributed_training_b200.parallel.state_dict import get_model_state_dict, load_model_state_dict
    cfg = tiny_config()
    m1, m2 = build_model(cfg.model), build_model(cfg.model)
    load_model_state_dict(m2, get_model_state_dict(m1, full=False), full=False)
    for a, b in zip(m1.parameters(), m2.parameters()):
        assert torch.equal(a, b)
