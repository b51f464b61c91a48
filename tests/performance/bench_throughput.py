"""Throughput / MFU of the training step for any config (run under torchrun).

    torchrun --nproc_per_node 8 tests/performance/bench_throughput.py --config config/llama2_7b_2d.yaml --tp-size 2

Same interface and output as the reference's ``tests/performance/bench_throughput.py``
(warm-up, timed loop of ``train_step``, tokens/s, per-GPU tokens/s, average MFU,
peak memory, ``--assert-min-mfu`` exits 2 below the gate); timing here is
CUDA events, max over ranks.
"""

from __future__ import annotations

import argparse
import json
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from build_your_own_distributed_training_b200.parallel.process_groups import destroy_distributed  # noqa: E402
from build_your_own_distributed_training_b200.training.loop import train_step  # noqa: E402
from build_your_own_distributed_training_b200.training.trainer import Trainer  # noqa: E402
from train import build_config  # noqa: E402


def main() -> None:
    p = argparse.ArgumentParser(description="Throughput benchmark.")
    p.add_argument("--config", required=True)
    p.add_argument("--tp-size", type=int, default=1)
    p.add_argument("--backend", type=str, default=None)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--gpu-type", type=str, default="b200")
    p.add_argument("--nccl-comm", action="store_true", help="collectives through NCCL instead of NVLink kernels")
    p.add_argument("--assert-min-mfu", type=float, default=None)
    a = p.parse_args()
    ns = argparse.Namespace(config=a.config, tp_size=a.tp_size, dp_size=None, backend=a.backend,
                            run_id="bench_tput", resume_from=None, max_steps=None)
    cfg = build_config(ns)
    cfg.eval_interval = cfg.save_interval = cfg.profile_steps = 0
    cfg.log_interval = 10 ** 9
    cfg.kernels.fused_comm = not a.nccl_comm
    tr = Trainer(cfg, gpu_type=a.gpu_type)
    ctx = tr.ctx
    try:
        def step():
            w, _ = tr._next_window()
            return train_step(tr.model, w, tr.optimizer, tr.scheduler, ctx, cfg, gpu_type=a.gpu_type)
        for _ in range(a.warmup):
            step()
        cuda = ctx.device.type == "cuda"
        if cuda:
            torch.cuda.reset_peak_memory_stats(ctx.device)
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
        import time
        t0 = time.perf_counter()
        mfu = 0.0
        for _ in range(a.steps):
            mfu += step().mfu or 0.0
        if cuda:
            e1.record()
            torch.cuda.synchronize()
            el = e0.elapsed_time(e1) / 1e3
        else:
            el = time.perf_counter() - t0
        t = torch.tensor([el], device=ctx.device)
        if dist.is_initialized():
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        tokens = cfg.data.micro_batch_size * cfg.data.seq_len * cfg.grad_accum_steps * ctx.dims.dp_size * a.steps
        tps = tokens / float(t)
        if ctx.is_rank0:
            print(json.dumps({"event": "bench_throughput", "tp_size": ctx.dims.tp_size, "dp_size": ctx.dims.dp_size,
                              "world_size": ctx.world_size, "tokens_per_sec": round(tps, 1),
                              "tokens_per_sec_per_gpu": round(tps / ctx.world_size, 1),
                              "avg_mfu": round(mfu / a.steps, 4),
                              "peak_mem_mb": round(torch.cuda.max_memory_allocated(ctx.device) / 1e6, 1)
                              if cuda else 0.0, "steps": a.steps}))
        if a.assert_min_mfu is not None and mfu / a.steps < a.assert_min_mfu:
            if ctx.is_rank0:
                print(f"FAIL: MFU {mfu / a.steps:.4f} < threshold {a.assert_min_mfu}", file=sys.stderr)
            sys.exit(2)
    finally:
        destroy_distributed()


if __name__ == "__main__":
    main()
