"""Throughput, MFU, loss aggregation and memory metrics.

Formulas follow ``src/observability/metrics.py:46-178``: FLOPs per token
``6 N + 12 L d max_seq_len``, MFU over all GPUs of the job, loss averaged over
dp.  Additions: a ``b200`` peak (the measured cuBLAS bf16 figure when
``MEASURED_PEAKS.json`` sits at the repository root, else NVIDIA's dense
bf16 figure), an MFU variant that uses the trained ``seq_len`` in the attention
term (the reference always uses ``max_seq_len``), and device-time fields.
"""

from __future__ import annotations

import json
import os
from dataclasses import dataclass

import torch
import torch.distributed as dist

from ..config import ModelConfig

B200_DENSE_BF16_TFLOPS = 2250.0


def _b200_peak() -> float:
    here = os.path.dirname(os.path.abspath(__file__))
    path = os.path.join(here, "..", "..", "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["bf16_tflops"])
    except (OSError, KeyError, ValueError):
        return B200_DENSE_BF16_TFLOPS


PEAK_TFLOPS_BF16: dict[str, float] = {
    "a100": 312.0, "a100-80gb": 312.0, "h100": 989.0, "h100-sxm": 989.0, "v100": 125.0,
    "b200": _b200_peak(), "b200-spec": B200_DENSE_BF16_TFLOPS, "cpu": 1.0,
}


@dataclass
class StepMetrics:
    loss: float
    grad_norm: float
    learning_rate: float
    tokens_per_second: float
    step_time_s: float
    data_wait_s: float
    mfu: float | None
    peak_memory_bytes: int
    device_time_s: float | None = None

    def perplexity(self) -> float:
        return float(torch.exp(torch.tensor(min(self.loss, 20.0))))


def aggregate_loss(local_loss: torch.Tensor, dp_group: dist.ProcessGroup | None) -> float:
    v = local_loss.detach().clone().float()
    if dist.is_initialized() and dp_group is not None and dist.get_world_size(dp_group) > 1:
        dist.all_reduce(v, group=dp_group)
        v /= dist.get_world_size(dp_group)
    return float(v.item())


def estimate_flops_per_token(config: ModelConfig, seq_len: int | None = None) -> float:
    """``6 N + 12 L d S``; ``S`` is ``max_seq_len`` unless ``seq_len`` is given."""
    s = config.max_seq_len if seq_len is None else seq_len
    return float(6 * config.num_parameters() + 12 * config.n_layers * config.d_model * s)


def compute_mfu(tokens_per_second: float, flops_per_token: float, num_gpus: int,
                gpu_type: str) -> float | None:
    peak = PEAK_TFLOPS_BF16.get(gpu_type.lower())
    if peak is None:
        return None
    return tokens_per_second * flops_per_token / (peak * 1e12 * num_gpus)


def compute_throughput(num_tokens: int, elapsed_seconds: float) -> float:
    return num_tokens / elapsed_seconds if elapsed_seconds > 0 else 0.0


def reset_peak_memory(device: torch.device) -> None:
    if device.type == "cuda":
        torch.cuda.reset_peak_memory_stats(device)


def peak_memory_bytes(device: torch.device) -> int:
    return int(torch.cuda.max_memory_allocated(device)) if device.type == "cuda" else 0
