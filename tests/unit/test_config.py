import pytest

from build_your_own_distributed_training_b200.config import ModelConfig, TrainingConfig
from tests.helpers import ROOT, TINY


def test_yaml_roundtrip_and_tuple_betas():
    cfg = TrainingConfig.from_yaml(TINY)
    assert cfg.model.n_layers == 2 and cfg.model.n_kv_heads == 2
    assert isinstance(cfg.optimizer.betas, tuple)
    again = TrainingConfig.from_dict(cfg.to_dict())
    assert again == cfg


@pytest.mark.parametrize("name", ["base", "125m", "7b", "test_tiny", "llama2_7b_2d", "llama2_7b_fsdp",
                                  "llama3_8b_tp8", "llama_125m_tp2dp4"])
def test_shipped_configs_parse(name):
    TrainingConfig.from_yaml(f"{ROOT}/config/{name}.yaml")


def test_unknown_key_raises():
    with pytest.raises(TypeError, match="Unknown config key 'lerning_rate'"):
        TrainingConfig.from_dict({"optimizer": {"lerning_rate": 1.0}})


def test_model_defaults():
    m = ModelConfig(d_model=768, n_heads=12)
    assert m.n_kv_heads == 12
    assert m.ffn_hidden_size == 2048  # 8/3*768 = 2048 rounded up to 256
    assert m.head_dim == 64
    m7 = ModelConfig(vocab_size=32000, d_model=4096, n_layers=32, n_heads=32, ffn_hidden_size=11008,
                     tie_embeddings=False)
    assert m7.num_parameters() == 6_738_149_376


def test_validate_global_batch():
    cfg = TrainingConfig.from_yaml(TINY)
    cfg.validate(world_size=4, dp_size=2, tp_size=2)
    assert cfg.data.global_batch_size == 4 * 2 * 2
    cfg.data.global_batch_size = 7
    with pytest.raises(ValueError, match="global_batch_size=7"):
        cfg.validate(world_size=4, dp_size=2, tp_size=2)


def test_validate_tp_divisibility():
    cfg = TrainingConfig.from_yaml(TINY)  # 2 kv heads
    with pytest.raises(ValueError, match="n_kv_heads=2 is not divisible by tp_size=4"):
        cfg.validate(world_size=4, dp_size=1, tp_size=4)


def test_validate_strategy():
    cfg = TrainingConfig.from_yaml(TINY)
    cfg.parallel.sharding_strategy = "ZERO9"
    with pytest.raises(ValueError, match="sharding_strategy"):
        cfg.validate(1, 1, 1)
