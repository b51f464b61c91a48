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
    # its gradient-norm partials: weight 1 below the split, rep_w above (TP-replicated entries)
    part = torch.zeros(native().reduce_scatter_blocks(n) + 3, device=dev)
    split = n // 3 + 1
    pc.reduce_scatter_mean(out, grad, world, part=part, split=split, rep_w=0.5)
    wts = torch.ones(n, device=dev, dtype=torch.float64)
    wts[split:] = 0.5
    ref_ss = float((out.double() ** 2 * wts).sum())
    check(abs(float(part.double().sum()) - ref_ss) < 1e-5 * ref_ss, "reduce-scatter norm partials differ from fp64")
    check(float(part[-3:].abs().sum()) == 0.0, "reduce-scatter wrote past its blocks")

    # ---- TP transport
    M, K, N = max(1024, 256 * world), 512, 768  # 256-row slices per rank for the fused SP GEMMs
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
    # sequence parallelism: all-gather fused in front of the GEMM, dgrad fused with the reduce-scatter
    xl = torch.randn(M // world, K, device=dev).to(torch.bfloat16)
    for it in range(2):
        y, xg = tpc.gather_gemm(xl, w[:N], 0)
        ref_g = torch.empty(M, K, device=dev, dtype=torch.bfloat16)
        dist.all_gather_into_tensor(ref_g, xl)
        check(torch.equal(xg, ref_g), f"fused all-gather GEMM: gathered rows differ (call {it})")
        check(rel(y, gemm.mm_nt(ref_g, w)) < 1e-2, f"fused all-gather GEMM mismatch (call {it})")
        dy = torch.randn(M, N, device=dev).to(torch.bfloat16)
        dxl = tpc.dgrad_reduce_scatter(dy, w)
        full = gemm.mm_nn(dy, w).float()
        ref_rs = torch.empty(M // world, K, device=dev)
        dist.reduce_scatter_tensor(ref_rs, full)
        check(rel(dxl, ref_rs) < 1e-2, f"fused dgrad reduce-scatter mismatch (call {it})")
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
    # (tp, sequence parallel, loss parallel): pure TP, TP+SP, pure ZeRO, vocabulary-parallel loss,
    # and at 4+ GPUs the 2-D layout tp2 x dp(world/2), where the ZeRO pull transport and the
    # TP-fused GEMMs run in the same step
    layouts = [(world, False, False, "FULL_SHARD"), (world, True, False, "FULL_SHARD"),
               (1, False, False, "FULL_SHARD"), (world, False, True, "FULL_SHARD"),
               (1, False, False, "NO_SHARD"), (1, False, False, "HYBRID_SHARD")]
    if world >= 4:
        layouts += [(2, False, False, "FULL_SHARD"), (2, True, True, "FULL_SHARD"), (2, False, False, "NO_SHARD")]
    for tp, sp, lp, strategy in layouts:
        ctx = build_process_context(tp, backend="nccl", verbose=False)
        for fused in (True, False):
            cfg = TrainingConfig.from_yaml(os.path.join(root, "config", "test_tiny.yaml"))
            cfg.model.vocab_size, cfg.model.d_model, cfg.model.n_layers = 1024, 512, 2
            # 4 KV heads up to tp = 4; at tp = 8 every rank needs one of its own
            cfg.model.n_heads, cfg.model.n_kv_heads, cfg.model.ffn_hidden_size = 8, max(4, tp), 1024
            # 1024 tokens per step: 256-row slices per rank up to tp=4, so sequence parallelism
            # takes the fused all-gather GEMM and dgrad reduce-scatter paths
            cfg.model.max_seq_len = 512
            cfg.data.seq_len, cfg.data.micro_batch_size, cfg.data.dataset_path = 512, 2, "uniform"
            cfg.parallel.tp_size = tp
            cfg.parallel.sequence_parallel = sp
            cfg.parallel.loss_parallel = lp
            cfg.parallel.sharding_strategy = strategy
            cfg.parallel.param_dtype = "bfloat16"
            cfg.backend = "nccl"
            cfg.kernels.fused_comm = fused
            cfg.eval_interval = cfg.save_interval = 0
            cfg.log_interval = 10 ** 9
            tr = Trainer(cfg, ctx=ctx, gpu_type="b200")
            steps = []
            for _ in range(3):
                wdw, _ = tr._next_window()
                m = train_step(tr.model, wdw, tr.optimizer, tr.scheduler, ctx, cfg)
                steps.append((m.loss, m.grad_norm))
            results[(tp, sp, lp, strategy, fused)] = steps
            # every rank reports the same loss and norm
            t = torch.tensor([v for st in steps for v in st], device=dev, dtype=torch.float64)
            every = [torch.empty_like(t) for _ in range(world)]
            dist.all_gather(every, t)
            check(all(torch.equal(every[0], e) for e in every),
                  f"tp={tp} sp={sp} lp={lp} {strategy} fused={fused}: ranks disagree")
        sf, sn = results[(tp, sp, lp, strategy, True)], results[(tp, sp, lp, strategy, False)]
        tag = f"tp={tp} sp={sp} lp={lp} {strategy}"
        for i, ((lf, gf), (ln, gn)) in enumerate(zip(sf, sn)):
            check(abs(lf - ln) < 1e-3 * (i + 1), f"{tag} step {i}: loss fused {lf} vs nccl {ln}")
            check(abs(gf - gn) < 1e-2 * max(1.0, gn), f"{tag} step {i}: grad norm {gf} vs {gn}")
    # the vocabulary-parallel loss equals the replicated-head loss on the same data
    for fused in (True, False):
        a, b = results[(world, False, True, "FULL_SHARD", fused)], results[(world, False, False, "FULL_SHARD", fused)]
        check(abs(a[0][0] - b[0][0]) < 1e-3, f"loss_parallel first loss {a[0][0]} vs replicated head {b[0][0]}")
    torch.cuda.synchronize()
    check(native().device_error() == 0, "device error word set after training")
    if rank == 0:
        print("MGPU_OK", results)
    symmetric.release_all()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
