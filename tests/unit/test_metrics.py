import io
import json

import torch

from build_your_own_distributed_training_b200.config import ModelConfig
from build_your_own_distributed_training_b200.observability.logging import build_logger
from build_your_own_distributed_training_b200.observability.metrics import (PEAK_TFLOPS_BF16, StepMetrics,
                                                                          aggregate_loss, compute_mfu,
                                                                          compute_throughput,
                                                                          estimate_flops_per_token)


def test_throughput_guard():
    assert compute_throughput(100, 0.0) == 0.0
    assert compute_throughput(100, 2.0) == 50.0


def test_flops_formula():
    m = ModelConfig(vocab_size=128, d_model=64, n_layers=2, n_heads=4, max_seq_len=32)
    assert estimate_flops_per_token(m) == 6 * m.num_parameters() + 12 * 2 * 64 * 32
    assert estimate_flops_per_token(m, seq_len=16) == 6 * m.num_parameters() + 12 * 2 * 64 * 16


def test_mfu_by_hand_and_unknown_gpu():
    assert abs(compute_mfu(1.6e5, 6e9, 8, "a100") - 1.6e5 * 6e9 / (312e12 * 8)) < 1e-12
    assert compute_mfu(1.0, 1.0, 1, "tpu-v9") is None
    assert PEAK_TFLOPS_BF16["b200"] > 1000


def test_aggregate_without_group_and_ppl():
    assert aggregate_loss(torch.tensor(2.5), None) == 2.5
    m = StepMetrics(100.0, 0, 0, 0, 0, 0, None, 0)
    assert abs(m.perplexity() - float(torch.exp(torch.tensor(20.0)))) < 1


def test_log_schema_and_gating():
    buf = io.StringIO()
    build_logger(0, "r", buf).metric("step", step=3, loss=1.5)
    rec = json.loads(buf.getvalue())
    assert {"ts", "level", "rank", "run_id", "event"} <= set(rec) and rec["step"] == 3
    buf2 = io.StringIO()
    lg = build_logger(1, "r", buf2)
    lg.info("x")
    assert buf2.getvalue() == ""
    lg.warning("w")
    assert json.loads(buf2.getvalue())["level"] == "WARNING"
