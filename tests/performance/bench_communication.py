"""Communication share of CUDA time, NVLink kernels vs NCCL, prefetch on vs off.

    torchrun --nproc_per_node 8 tests/performance/bench_communication.py --config config/llama2_7b_2d.yaml --tp-size 2

Same idea as the reference's ``tests/performance/bench_communication.py``
(profiler window, communication fraction by kernel name).  Fused
GEMM+collective kernels are reported separately: their time cannot be split
into compute and communication by name.
"""

from __future__ import annotations

import argparse
import json
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))

import torch  # noqa: E402
from torch.profiler import ProfilerActivity, profile  # noqa: E402

from build_your_own_distributed_training_b200.observability.profiler import communication_fraction  # noqa: E402
from build_your_own_distributed_training_b200.parallel.process_groups import destroy_distributed  # noqa: E402
from build_your_own_distributed_training_b200.training.loop import train_step  # noqa: E402
from build_your_own_distributed_training_b200.training.trainer import Trainer  # noqa: E402
from train import build_config  # noqa: E402


def run(cfg, steps: int) -> dict:
    tr = Trainer(cfg, gpu_type="b200")

    def step():
        w, _ = tr._next_window()
        return train_step(tr.model, w, tr.optimizer, tr.scheduler, tr.ctx, cfg, gpu_type="b200")
    for _ in range(3):
        step()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(steps):
            m = step()
        torch.cuda.synchronize()
    b = communication_fraction(prof)
    return {"tok_per_s": round(m.tokens_per_second, 1), "comm_fraction": round(b.comm_fraction, 4),
            "fused_comm_gemm_us": round(b.fused_cuda_us, 1), "total_cuda_us": round(b.total_cuda_us, 1)}


def main() -> None:
    p = argparse.ArgumentParser()
    p.add_argument("--config", required=True)
    p.add_argument("--tp-size", type=int, default=1)
    p.add_argument("--steps", type=int, default=2)
    a = p.parse_args()
    out = {}
    try:
        for label, fused, prefetch in (("nvlink+prefetch", True, True), ("nccl+prefetch", False, True),
                                       ("nvlink,no-prefetch", True, False)):
            ns = argparse.Namespace(config=a.config, tp_size=a.tp_size, dp_size=None, backend=None,
                                    run_id="bench_comm", resume_from=None, max_steps=None)
            cfg = build_config(ns)
            cfg.eval_interval = cfg.save_interval = cfg.profile_steps = 0
            cfg.log_interval = 10 ** 9
            cfg.kernels.fused_comm = fused
            cfg.parallel.forward_prefetch = prefetch
            out[label] = run(cfg, a.steps)
        if int(os.environ.get("RANK", "0")) == 0:
            print(json.dumps({"event": "bench_communication", **out}))
    finally:
        destroy_distributed()


if __name__ == "__main__":
    main()
