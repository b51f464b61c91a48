"""Multi-GPU checks of the NVLink transport, run by test_multi_gpu.py under torchrun.

Every peer-memory collective is compared with NCCL on the same data, and the
fused row-parallel GEMM + all-reduce with a GEMM followed by an NCCL
all-reduce; TP ranks must agree bit for bit.
"""

import os
import sys
from datetime import timedelta

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))

from build_your_own_distributed_training_b200.ops import gemm  # noqa: E402
from build_your_own_distributed_training_b200.ops._ext import native  # noqa: E402
from build_your_own_distributed_training_b200.parallel import symmetric  # noqa: E402


def rel(a, b):
    return float((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12))


def check(cond, msg):
    if not cond:
        raise AssertionError(msg)


def main():
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    rank, world = dist.get_rank(), dist.get_world_size()
    dev = torch.device("cuda", local)
    g = dist.group.WORLD
    torch.manual_seed(1234 + rank)

    # ---- ZeRO transport
    pc = symmetric.PeerComm(g, dev)
    n = 4096 * 33
    shard, grad = pc.alloc_many([(n, torch.bfloat16), (n * world, torch.float32)])
    shard.copy_(torch.randn(n, device=dev).to(torch.bfloat16))
    grad.copy_(torch.randn(n * world, device=dev))
    pc.barrier()
    full = torch.empty(n * world, device=dev, dtype=torch.bfloat16)
    pc.all_gather(full, shard)
    ref = torch.empty_like(full)
    dist.all_gather_into_tensor(ref, shard.clone())
    check(torch.equal(full, ref), "peer all-gather differs from NCCL")
    out = torch.empty(n, device=dev)
    pc.reduce_scatter_mean(out, grad, world)
    every = [torch.empty_like(grad) for _ in range(world)]
    dist.all_gather(every, grad.clone())
    exact = sum(e[rank * n:(rank + 1) * n] for e in every) / world  # same order: rank 0..world-1
    check(torch.equal(out, exact), "peer reduce-scatter is not the fixed-order sum")

    # ---- TP transport
    M, K, N = 1024, 512, 768
    tpc = symmetric.TPComm(g, dev, M, N)
    x = torch.randn(M, K, device=dev).to(torch.bfloat16)
    w = (torch.randn(N, K, device=dev) * 0.05).to(torch.bfloat16)
    gen = torch.Generator(device=dev).manual_seed(7)  # the residual stream is replicated across TP ranks
    res = torch.randn(M, N, device=dev, generator=gen).to(torch.bfloat16)
    for it in range(3):  # repeated calls exercise both staging slots and the epochs
        y = tpc.gemm_all_reduce(x, w, res)
        part = gemm.mm_nt(x, w)
        dist.all_reduce(part)
        check(rel(y, part.float() + res.float()) < 1e-2, f"fused GEMM+all-reduce mismatch (call {it})")
        ys = [torch.empty_like(y) for _ in range(world)]
        dist.all_gather(ys, y)
        check(all(torch.equal(ys[0], t) for t in ys), "TP ranks disagree after the fused all-reduce")
    # fused GEMM -> reduce-scatter of rows (sequence parallelism), residual in the scattered layout
    rows = M // world
    res_rs = torch.randn(rows, N, device=dev).to(torch.bfloat16)
    for it in range(3):
        y = tpc.gemm_reduce_scatter(x, w, res_rs)
        part = gemm.mm_nt(x, w).float()
        ref = torch.empty(rows, N, device=dev)
        dist.reduce_scatter_tensor(ref, part)
        check(rel(y, ref + res_rs.float()) < 1e-2, f"fused GEMM+reduce-scatter mismatch (call {it})")
    a = torch.randn(M, N, device=dev).to(torch.bfloat16)
    ar = tpc.all_reduce(a)
    ref_ar = a.float().clone()
    dist.all_reduce(ref_ar)
    check(rel(ar, ref_ar) < 1e-2, "peer all-reduce mismatch")
    ag = tpc.all_gather_rows(a[:M // world])
    ref_ag = torch.empty_like(ag)
    dist.all_gather_into_tensor(ref_ag, a[:M // world].contiguous())
    check(torch.equal(ag, ref_ag), "peer all-gather rows mismatch")
    rs = tpc.reduce_scatter_rows(a)
    ref_rs = torch.empty(M // world, N, device=dev)
    dist.reduce_scatter_tensor(ref_rs, a.float())
    check(rel(rs, ref_rs) < 1e-2, "peer reduce-scatter rows mismatch")
    torch.cuda.synchronize()
    check(native().device_error() == 0, "device error word set")

    # ---- engine: fused transport vs NCCL transport, same seeds and data
    from build_your_own_distributed_training_b200.config import TrainingConfig
    from build_your_own_distributed_training_b200.parallel.process_groups import build_process_context
    from build_your_own_distributed_training_b200.training.loop import train_step
    from build_your_own_distributed_training_b200.training.trainer import Trainer
    root = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    results = {}
    for tp, sp in ((world, False), (world, True), (1, False)):
        ctx = build_process_context(tp, backend="nccl", verbose=False)
        for fused in (True, False):
            cfg = TrainingConfig.from_yaml(os.path.join(root, "config", "test_tiny.yaml"))
            cfg.model.vocab_size, cfg.model.d_model, cfg.model.n_layers = 1024, 512, 2
            cfg.model.n_heads, cfg.model.n_kv_heads, cfg.model.ffn_hidden_size = 8, 4, 1024
            cfg.model.max_seq_len = 256
            cfg.data.seq_len, cfg.data.micro_batch_size, cfg.data.dataset_path = 256, 2, "uniform"
            cfg.parallel.tp_size = tp
            cfg.parallel.sequence_parallel = sp
            cfg.parallel.param_dtype = "bfloat16"
            cfg.backend = "nccl"
            cfg.kernels.fused_comm = fused
            cfg.eval_interval = cfg.save_interval = 0
            cfg.log_interval = 10 ** 9
            tr = Trainer(cfg, ctx=ctx, gpu_type="b200")
            losses = []
            for _ in range(3):
                wdw, _ = tr._next_window()
                losses.append(train_step(tr.model, wdw, tr.optimizer, tr.scheduler, ctx, cfg).loss)
            results[(tp, sp, fused)] = losses
        lf, ln = results[(tp, sp, True)], results[(tp, sp, False)]
        check(all(abs(p - q) < 2e-2 for p, q in zip(lf, ln)), f"tp={tp} sp={sp}: fused {lf} vs nccl {ln}")
    torch.cuda.synchronize()
    check(native().device_error() == 0, "device error word set after training")
    if rank == 0:
        print("MGPU_OK", results)
    symmetric.release_all()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
