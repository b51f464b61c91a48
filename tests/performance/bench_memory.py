"""Peak memory vs sequence length, with and without activation checkpointing.

    python tests/performance/bench_memory.py --config config/llama2_7b_2d.yaml --layers 4

Same sweep as the reference's ``tests/performance/bench_memory.py``.
"""

from __future__ import annotations

import argparse
import json
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))

import torch  # noqa: E402

from build_your_own_distributed_training_b200.parallel.process_groups import destroy_distributed  # noqa: E402
from build_your_own_distributed_training_b200.training.loop import train_step  # noqa: E402
from build_your_own_distributed_training_b200.training.trainer import Trainer  # noqa: E402
from train import build_config  # noqa: E402


def main() -> None:
    p = argparse.ArgumentParser()
    p.add_argument("--config", required=True)
    p.add_argument("--layers", type=int, default=None, help="override n_layers (memory scales per layer)")
    p.add_argument("--seq-lens", type=str, default="1024,2048,4096")
    a = p.parse_args()
    rows = []
    try:
        for seq in (int(s) for s in a.seq_lens.split(",")):
            for ac in (False, True):
                ns = argparse.Namespace(config=a.config, tp_size=1, dp_size=None, backend=None, run_id="bench_mem",
                                        resume_from=None, max_steps=None)
                cfg = build_config(ns)
                cfg.eval_interval = cfg.save_interval = cfg.profile_steps = 0
                cfg.log_interval = 10 ** 9
                cfg.parallel.tp_size = 1
                cfg.data.seq_len = seq
                cfg.model.max_seq_len = max(cfg.model.max_seq_len, seq)
                cfg.parallel.activation_checkpointing = ac
                if a.layers:
                    cfg.model.n_layers = a.layers
                tr = Trainer(cfg, gpu_type="b200")
                w, _ = tr._next_window()
                torch.cuda.reset_peak_memory_stats()
                train_step(tr.model, w, tr.optimizer, tr.scheduler, tr.ctx, cfg)
                rows.append({"seq_len": seq, "activation_checkpointing": ac,
                             "peak_mem_mb": round(torch.cuda.max_memory_allocated() / 1e6, 1)})
                del tr
                torch.cuda.empty_cache()
        print(json.dumps({"event": "bench_memory", "rows": rows}))
    finally:
        destroy_distributed()


if __name__ == "__main__":
    main()
