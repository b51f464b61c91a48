"""The GPU path (sharding engine + native kernels) against the CPU fp32 model."""

from __future__ import annotations

import copy

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a GPU", allow_module_level=True)

from build_your_own_distributed_training_b200.config import ModelConfig, ParallelConfig  # noqa: E402
from build_your_own_distributed_training_b200.models.transformer import TransformerBlock, build_model  # noqa: E402
from build_your_own_distributed_training_b200.ops._ext import native  # noqa: E402
from build_your_own_distributed_training_b200.parallel.fsdp import FullyShardedModel  # noqa: E402
from build_your_own_distributed_training_b200.training.grad_utils import device_clip_state, sharded_total_norm  # noqa: E402
from build_your_own_distributed_training_b200.training.optimizer import ShardedAdamW  # noqa: E402

DEV = torch.device("cuda", 0)


def _cfg(tie: bool) -> ModelConfig:
    return ModelConfig(vocab_size=1024, d_model=512, n_layers=2, n_heads=8, n_kv_heads=2, ffn_hidden_size=768,
                       max_seq_len=256, tie_embeddings=tie)


def _engine(model):
    eng = FullyShardedModel(model, None, ParallelConfig(), {TransformerBlock}, device=DEV)
    model.rope_cos, model.rope_sin = model.rope_cos.to(DEV), model.rope_sin.to(DEV)
    return eng


@pytest.mark.parametrize("tie", [False, True])
def test_loss_and_grads_match_cpu_fp32(tie):
    torch.manual_seed(0)
    cpu = build_model(_cfg(tie))
    gpu_model = copy.deepcopy(cpu)
    eng = _engine(gpu_model)
    tok = torch.randint(0, 1024, (2, 256))
    lab = torch.randint(0, 1024, (2, 256))
    _, ref = cpu(tok, labels=lab)
    ref.backward()
    _, loss = eng(tok.to(DEV), labels=lab.to(DEV))
    loss.backward()
    eng.wait_reduce()
    torch.cuda.synchronize()
    assert abs(float(loss) - float(ref)) < 2e-2
    named = dict(cpu.named_parameters())
    for u in eng.units:
        for e in u.entries:
            g_ref = named[e.fqn].grad
            g = u.grad_shard[e.offset:e.offset + e.numel].view(e.shape).cpu()
            rel = float((g - g_ref).norm() / g_ref.norm().clamp_min(1e-12))
            assert rel < 6e-2, (e.fqn, rel)
    assert native().device_error() == 0


def test_training_reduces_loss():
    torch.manual_seed(0)
    model = build_model(_cfg(False))
    eng = _engine(model)
    model.return_logits = False
    opt = ShardedAdamW(eng, lr=3e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)
    g = torch.Generator().manual_seed(1)
    base = torch.randint(0, 64, (4, 257), generator=g)  # small alphabet: learnable
    tok, lab = base[:, :-1].to(DEV), base[:, 1:].to(DEV)
    losses = []
    for _ in range(30):
        opt.zero_grad()
        _, loss = eng(tok, labels=lab)
        loss.backward()
        eng.wait_reduce()
        norm = sharded_total_norm(eng)
        opt.set_clip_state(device_clip_state(norm, 1.0))
        opt.step()
        losses.append(float(loss))
    assert losses[-1] < losses[0] - 2.0, losses
    assert native().device_error() == 0


def test_tiny_config_model_trains_on_gpu():
    """config/test_tiny.yaml's model (head_dim 16, seq 32) on the GPU kernels: first loss and
    gradients match the CPU fp32 model, and training lowers the loss."""
    import os

    from build_your_own_distributed_training_b200.config import TrainingConfig
    root = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    tcfg = TrainingConfig.from_yaml(os.path.join(root, "config", "test_tiny.yaml"))
    assert tcfg.model.head_dim == 16
    torch.manual_seed(0)
    cpu = build_model(tcfg.model)
    model = copy.deepcopy(cpu)
    eng = _engine(model)
    g = torch.Generator().manual_seed(3)
    S = tcfg.data.seq_len
    base = torch.randint(0, 32, (tcfg.data.micro_batch_size, S + 1), generator=g)
    tok, lab = base[:, :-1], base[:, 1:]
    _, ref = cpu(tok, labels=lab)
    _, loss = eng(tok.to(DEV), labels=lab.to(DEV))
    assert abs(float(loss) - float(ref)) < 2e-2
    model.return_logits = False
    opt = ShardedAdamW(eng, lr=3e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)
    losses = []
    for _ in range(40):
        opt.zero_grad()
        _, loss = eng(tok.to(DEV), labels=lab.to(DEV))
        loss.backward()
        eng.wait_reduce()
        opt.set_clip_state(device_clip_state(sharded_total_norm(eng), 1.0))
        opt.step()
        losses.append(float(loss))
    assert losses[-1] < losses[0] - 1.0, losses
    assert native().device_error() == 0
