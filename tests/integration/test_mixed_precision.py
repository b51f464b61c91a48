import torch

from build_your_own_distributed_training_b200.config import ParallelConfig
from build_your_own_distributed_training_b200.models.transformer import build_model
from build_your_own_distributed_training_b200.utils.dtype import autocast_dtype, build_mixed_precision, resolve_dtype
from tests.helpers import tiny_config


def test_policy_defaults_and_aliases():
    pol = build_mixed_precision(ParallelConfig())
    assert pol.param_dtype == torch.bfloat16 and pol.reduce_dtype == torch.float32
    assert autocast_dtype(ParallelConfig(param_dtype="fp32")) == torch.float32
    for a, b in (("bf16", "bfloat16"), ("fp16", "half"), ("fp32", "float")):
        assert resolve_dtype(a) == resolve_dtype(b)


def test_cpu_autocast_bf16_with_fp32_master():
    cfg = tiny_config()
    m = build_model(cfg.model)
    tok = torch.randint(0, 256, (2, 16))
    with torch.autocast("cpu", dtype=torch.bfloat16):
        _, loss = m(tok, labels=tok)
    loss.backward()
    assert all(p.dtype == torch.float32 for p in m.parameters())
    assert torch.isfinite(loss)
