"""Throughput benchmark: LLaMA-2-7B shape, 2-D (tp x dp) training step on B200s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl native|reference]
    torchrun --nproc-per-node N --master-addr 127.0.0.1 bench.py --gpus N ...

Workload (weak scaling, 4096 tokens per GPU per step, uniform-random tokens,
random-init weights, bf16 compute, fp32 master + AdamW, full optimizer step
every step):

    N=1: tp=1 dp=1 micro-batch 1      N=2: tp=2 dp=1 micro-batch 2
    N=4: tp=2 dp=2 micro-batch 2      N=8: tp=2 dp=4 micro-batch 2 (headline)

Model: 32 layers, d_model 4096, 32 heads (MHA), SwiGLU 11008, vocab 32000,
seq 4096, untied head.  Every timed step goes through the public
``train_step`` API: the micro-batch is copied host->device from pinned memory,
forward/backward/clip/AdamW run, and the loss/grad-norm are read back.

``value`` is tokens/s from CUDA events around the K timed steps (barrier +
synchronize on both sides, max elapsed over ranks).  ``e2e`` is the same loop
timed by the host clock.  ``--impl reference`` runs the unmodified reference
(installed under baseline/_ref) through its own ``Trainer``/``train_step`` on
the same workload, timed the same way.
"""

from __future__ import annotations

import argparse
import contextlib
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
SEQ = 4096
MODEL = dict(vocab_size=32000, d_model=4096, n_layers=32, n_heads=32, n_kv_heads=32,
             ffn_hidden_size=11008, max_seq_len=4096, rope_theta=10000.0, norm_eps=1e-5,
             tie_embeddings=False, dropout=0.0, attention_bias=False, mlp_bias=False)
METRIC = "7B FSDP×TP tokens/s & MFU (max over ranks) at 1/2/4/8 B200 vs ref NCCL"


def topology(n: int) -> tuple[int, int, int]:
    """(tp, dp, micro_batch) for n GPUs."""
    if n == 1:
        return 1, 1, 1
    return 2, n // 2, 2


def flops_per_token() -> float:
    d, L, V, F = MODEL["d_model"], MODEL["n_layers"], MODEL["vocab_size"], MODEL["ffn_hidden_size"]
    n_params = V * d + L * (4 * d * d + 3 * d * F) + V * d
    return 6.0 * n_params + 12.0 * L * d * MODEL["max_seq_len"]


def peak_tflops(key: str = "bf16_tflops") -> float:
    """Measured cuBLAS bf16 peak: ``bf16_tflops`` (burst) or ``bf16_tflops_sustained``
    (a seconds-long loop under the power cap, the fair peak for a long training step)."""
    fallback = {"bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}[key]
    try:
        with open(os.path.join(HERE, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)[key])
    except (OSError, KeyError, ValueError):
        return fallback


class ClockSampler:
    """nvidia-smi sampling every 200 ms while the timed region runs (rank 0)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, enabled: bool) -> None:
        self.enabled = enabled
        self.proc = None
        self.path = None

    def __enter__(self):
        if self.enabled:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            try:
                self.proc = subprocess.Popen(
                    ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                     "-lms", "200", "-f", self.path], stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
            except OSError:
                self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self, n_gpus: int) -> dict:
        if not self.path or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as f:
            for line in f:
                p = [x.strip() for x in line.split(",")]
                if len(p) < 9 or not p[0].isdigit() or int(p[0]) >= n_gpus:
                    continue
                try:
                    sm.append(float(p[1]))
                    mx.append(float(p[2]))
                except ValueError:
                    continue
                for name, val in zip(names, p[5:9]):
                    if val.lower() == "active":
                        reasons.add(name)
        os.unlink(self.path)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def init_dist(n: int) -> tuple[int, int]:
    if n > 1 or "RANK" in os.environ:
        from datetime import timedelta
        local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(local)
        if not dist.is_initialized():
            dist.init_process_group("nccl", timeout=timedelta(seconds=600),
                                    device_id=torch.device("cuda", local))
        return dist.get_rank(), dist.get_world_size()
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", str(29400 + os.getpid() % 1000))
    os.environ.setdefault("RANK", "0")
    os.environ.setdefault("WORLD_SIZE", "1")
    os.environ.setdefault("LOCAL_RANK", "0")
    torch.cuda.set_device(0)
    return 0, 1


def timed_loop(step_fn, steps: int, world: int) -> tuple[float, float]:
    """Run ``steps`` calls; returns (device seconds, host seconds), each max over ranks."""
    if dist.is_initialized():
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    e0.record()
    for _ in range(steps):
        step_fn()
    e1.record()
    torch.cuda.synchronize()
    t1 = time.perf_counter()
    if dist.is_initialized():
        dist.barrier()
    dev = torch.tensor([e0.elapsed_time(e1) / 1e3, t1 - t0], device="cuda", dtype=torch.float64)
    if dist.is_initialized() and world > 1:
        dist.all_reduce(dev, op=dist.ReduceOp.MAX)
    return float(dev[0]), float(dev[1])


KERNEL_CLASSES = (
    # (class, substrings) in match order; the first match wins
    ("gemm+collective", ()),  # tcgen05 GEMM with the peer epilogue, see observability.profiler
    ("gemm", ("gemm_tcgen05", "gemm", "cutlass", "nvjet", "sm100_xmma")),
    ("attention", ("attn_", "flash", "fmha", "sdpa", "cudnn")),
    ("optimizer", ("adamw", "sumsq", "sum_parts", "multi_tensor", "foreach")),
    ("collective", ("nccl", "peer_", "dev_barrier")),
    ("norm/rope/swiglu/ce/embedding", ("rmsnorm", "rope_", "swiglu", "ce_", "count_valid", "embedding",
                                       "reduce_partials")),
)


def profile_one_step(step_fn, prefixes: tuple[str, ...]) -> tuple[int, dict]:
    """Runs one extra (untimed) step under torch.profiler; returns the number of this
    package's kernel launches in it and the summed device time per kernel class (ms).
    Kernels on different streams overlap, so the classes can add up to more than the
    step's device time; ``step_ms`` is the step's own CUDA-event time."""
    from torch.profiler import ProfilerActivity, profile
    sys.path.insert(0, HERE)
    from build_your_own_distributed_training_b200.observability.profiler import is_fused_comm_kernel
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        e0.record()
        step_fn()
        e1.record()
        torch.cuda.synchronize()
    n = 0
    split: dict[str, float] = {}
    other: dict[str, float] = {}
    for e in prof.events():
        if e.device_type != torch.autograd.DeviceType.CUDA:
            continue
        if any(p in e.name for p in prefixes):
            n += 1
        low = e.name.lower()
        cls = "other"
        if is_fused_comm_kernel(e.name):
            cls = "gemm+collective"
        else:
            for name, keys in KERNEL_CLASSES[1:]:
                if any(k in low for k in keys):
                    cls = name
                    break
        ms = e.time_range.elapsed_us() / 1e3
        split[cls] = split.get(cls, 0.0) + ms
        if cls == "other":
            other[e.name[:60]] = other.get(e.name[:60], 0.0) + ms
    split = {k: round(v, 2) for k, v in sorted(split.items(), key=lambda kv: -kv[1])}
    split["step_ms"] = round(e0.elapsed_time(e1), 2)
    split["top_other"] = {k: round(v, 2) for k, v in sorted(other.items(), key=lambda kv: -kv[1])[:5]}
    return n, split


# ----------------------------------------------------------------------------- native
def run_native(args, n: int, rank: int, world: int) -> dict:
    sys.path.insert(0, HERE)
    from build_your_own_distributed_training_b200.config import TrainingConfig
    from build_your_own_distributed_training_b200.training.loop import train_step
    from build_your_own_distributed_training_b200.training.trainer import Trainer

    tp, dp, mb = topology(n)
    cfg = TrainingConfig.from_yaml(os.path.join(HERE, "config", "llama2_7b_2d.yaml"))
    for k, v in MODEL.items():
        setattr(cfg.model, k, v)
    cfg.parallel.tp_size = tp
    cfg.parallel.dp_size = dp
    cfg.data.micro_batch_size = mb
    cfg.data.global_batch_size = 0
    cfg.data.dataset_path = "uniform"
    cfg.data.num_workers = 0
    cfg.data.seq_len = SEQ
    cfg.grad_accum_steps = 1
    cfg.backend = "nccl"
    cfg.log_interval = 10 ** 9
    cfg.eval_interval = 0
    cfg.save_interval = 0
    cfg.profile_steps = 0
    cfg.kernels.fused_comm = not args.nccl_comm
    with contextlib.redirect_stdout(sys.stderr):
        trainer = Trainer(cfg, gpu_type="b200")
    ctx = trainer.ctx

    def step():
        window, wait = trainer._next_window()
        return train_step(trainer.model, window, trainer.optimizer, trainer.scheduler, ctx, cfg,
                          gpu_type="b200", data_wait_s=wait)

    for _ in range(args.warmup):
        step()
    with ClockSampler(rank == 0) as clk:
        dev_s, host_s = timed_loop(step, args.steps, world)
    launches, split = profile_one_step(step, ("gemm_tcgen05", "attn_", "rmsnorm_", "rope_", "swiglu_", "embedding_",
                                     "ce_", "count_valid", "adamw", "sumsq", "sum_parts",
                                     "reduce_partials", "peer_", "dev_barrier"))
    from build_your_own_distributed_training_b200.ops._ext import native
    err = native().device_error()
    if err:
        raise RuntimeError(f"device error word set: {err}")
    return dict(tp=tp, dp=dp, mb=mb, dev_s=dev_s, host_s=host_s, clocks=clk.summary(n),
                launches_per_step=launches, split=split,
                h2d=2 * mb * SEQ * 8, d2h=16,
                peak_mem=torch.cuda.max_memory_allocated())


# ----------------------------------------------------------------------------- reference
def write_tokens(path: str, n_tokens: int, vocab: int, seed: int) -> None:
    import numpy as np
    rng = np.random.default_rng(seed)
    rng.integers(0, vocab, size=n_tokens, dtype=np.uint16).tofile(path)


def run_reference(args, n: int, rank: int, world: int) -> dict:
    ref = os.path.join(HERE, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "src", "training")):
        raise SystemExit("reference not installed under baseline/_ref: run baseline/install_ref.sh "
                         "before copying the tree to the GPU box")
    sys.path.insert(0, ref)
    from src.config import TrainingConfig as RefConfig  # the reference's own package
    from src.training.loop import train_step as ref_train_step
    from src.training.trainer import Trainer as RefTrainer

    tp, dp, mb = topology(n)
    windows = (args.warmup + args.steps + 4) * mb * dp
    tok_path = os.path.join(tempfile.gettempdir(), f"bench_tokens_{windows}.bin")
    if rank == 0 and not os.path.exists(tok_path):
        write_tokens(tok_path + ".tmp", windows * SEQ + 1, MODEL["vocab_size"], 1234)
        os.replace(tok_path + ".tmp", tok_path)
    if dist.is_initialized():
        dist.barrier()
    raw = {
        "model": dict(MODEL),
        "parallel": {"tp_size": tp, "dp_size": dp, "sharding_strategy": "FULL_SHARD",
                     "sequence_parallel": False, "activation_checkpointing": False,
                     "param_dtype": "bfloat16", "reduce_dtype": "float32", "buffer_dtype": "bfloat16"},
        "optimizer": {"name": "adamw", "lr": 3e-4, "weight_decay": 0.1, "betas": [0.9, 0.95],
                      "eps": 1e-8, "fused": True},
        "scheduler": {"warmup_steps": 100, "max_steps": 1000, "min_lr": 3e-5},
        "data": {"dataset_path": tok_path, "seq_len": SEQ, "micro_batch_size": mb,
                 "global_batch_size": 0, "num_workers": 0, "shuffle": True, "tokenizer_name": ""},
        "grad_accum_steps": 1, "max_grad_norm": 1.0, "log_interval": 10 ** 9, "eval_interval": 0,
        "save_interval": 0, "profile_steps": 0, "backend": "nccl", "run_id": "bench_ref",
        "checkpoint_dir": tempfile.gettempdir(),
    }
    note = "adamw fused=True (the reference default)"
    for fused in (True, False):
        raw["optimizer"]["fused"] = fused
        cfg = RefConfig.from_dict(raw)
        with contextlib.redirect_stdout(sys.stderr):
            trainer = RefTrainer(cfg, gpu_type="h100")
        ctx = trainer.ctx

        def step():
            window, wait = trainer._next_window()
            return ref_train_step(trainer.model, window, trainer.optimizer, trainer.scheduler, ctx, cfg,
                                  gpu_type="h100", data_wait_s=wait)

        try:
            with contextlib.redirect_stdout(sys.stderr):
                step()
            break
        except RuntimeError as exc:
            # torch's fused AdamW rejects the mix of DTensor (TP-sharded) and plain
            # (replicated) parameters the reference's TP plan produces; its own
            # config offers fused=False, which runs the same code path otherwise
            if not fused or "mixed torch.Tensor and DTensor" not in str(exc):
                raise
            note = "adamw fused=False (fused AdamW raises on the reference's mixed DTensor/Tensor params)"
            del trainer, step
            import gc
            gc.collect()
            torch.cuda.empty_cache()
    with contextlib.redirect_stdout(sys.stderr):
        for _ in range(args.warmup - 1):
            step()
        with ClockSampler(rank == 0) as clk:
            dev_s, host_s = timed_loop(step, args.steps, world)
    return dict(tp=tp, dp=dp, mb=mb, dev_s=dev_s, host_s=host_s, clocks=clk.summary(n),
                launches_per_step=0, h2d=2 * mb * SEQ * 8, d2h=8, ref_optimizer=note,
                peak_mem=torch.cuda.max_memory_allocated())


def main() -> None:
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=("native", "reference"), default="native")
    p.add_argument("--nccl-comm", action="store_true", help="route collectives through NCCL")
    args = p.parse_args()
    n = args.gpus
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    rank, world = init_dist(n)
    if world != n:
        raise SystemExit(f"--gpus {n} but WORLD_SIZE={world}")
    out: dict
    try:
        res = run_native(args, n, rank, world) if args.impl == "native" else \
            run_reference(args, n, rank, world)
    except Exception as exc:  # noqa: BLE001
        if args.impl == "reference":
            if rank == 0:
                print(json.dumps({"impl": "reference", "unavailable": f"{type(exc).__name__}: {exc}"[:300]}))
            _teardown()
            return
        raise
    tp, dp, mb = res["tp"], res["dp"], res["mb"]
    tokens = dp * mb * SEQ * args.steps
    value = tokens / res["dev_s"]
    e2e = tokens / res["host_s"]
    mfu = value * flops_per_token() / (n * peak_tflops() * 1e12)
    mfu_sustained = value * flops_per_token() / (n * peak_tflops("bf16_tflops_sustained") * 1e12)
    out = {
        "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": n,
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1e3 * res["dev_s"] / args.steps, 2), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic uniform-random token ids, random-init weights",
        "mfu": round(mfu, 4),
        "mfu_vs_sustained_peak": round(mfu_sustained, 4),
        "config": {"model": "llama2-7b (L32 d4096 h32 MHA ffn11008 V32000 untied)",
                   "global_batch": dp * mb, "seq_len": SEQ,
                   "parallelism": f"tp{tp}dp{dp}", "micro_batch": mb,
                   "l2": "no flush: per-step working set (13.5 GB bf16 weights + activations) >> 126 MB L2",
                   "optimizer": "AdamW fp32 master, clip 1.0, every step"},
        "clocks": res["clocks"],
        "e2e": {"value": round(e2e, 1), "unit": "tokens/s", "h2d_bytes_per_step": res["h2d"],
                "d2h_bytes_per_step": res["d2h"]},
        "gpu_launches": res["launches_per_step"] * args.steps,
        "peak_mem_gb": round(res["peak_mem"] / 1e9, 1),
    }
    if res.get("split"):
        out["device_ms_by_kernel_class"] = res["split"]
    if args.impl == "reference":
        out["impl"] = "reference"
        out["config"]["optimizer"] = res["ref_optimizer"]
    if rank == 0:
        print(json.dumps(out), flush=True)
    _teardown()


def _teardown() -> None:
    try:
        from build_your_own_distributed_training_b200.parallel.process_groups import destroy_distributed
        destroy_distributed()
    except Exception:  # noqa: BLE001
        if dist.is_initialized():
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
