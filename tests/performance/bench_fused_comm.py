"""TP collectives on 2+ GPUs: fused GEMM+all-reduce vs GEMM + NCCL all-reduce, peer vs NCCL all-reduce.

    torchrun --nproc_per_node 2 tests/performance/bench_fused_comm.py
"""
import os, sys
sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
from datetime import timedelta
import torch, torch.distributed as dist
from build_your_own_distributed_training_b200.ops import gemm
from build_your_own_distributed_training_b200.parallel import symmetric
local = int(os.environ["LOCAL_RANK"]); torch.cuda.set_device(local)
dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
rank, world = dist.get_rank(), dist.get_world_size(); dev = torch.device("cuda", local)
def tm(f, it=20):
    for _ in range(3): f()
    torch.cuda.synchronize(); dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(it): f()
    e1.record(); torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) / it], device=dev); dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t)
M = 8192
tpc = symmetric.TPComm(dist.group.WORLD, dev, M, 4096)
for (K, N, label) in [(2048, 4096, "wo fwd"), (5504, 4096, "down fwd")]:
    x = torch.randn(M, K, device=dev).to(torch.bfloat16); w = (torch.randn(N, K, device=dev) * 0.02).to(torch.bfloat16)
    r = torch.randn(M, N, device=dev).to(torch.bfloat16)
    t_g = tm(lambda: gemm.mm_nt(x, w, residual=r))
    def nccl_path():
        y = gemm.mm_nt(x, w); dist.all_reduce(y); return y + r
    t_n = tm(nccl_path)
    t_f = tm(lambda: tpc.gemm_all_reduce(x, w, r))
    a = torch.randn(M, N, device=dev).to(torch.bfloat16)
    t_ar_n = tm(lambda: dist.all_reduce(a))
    t_ar_p = tm(lambda: tpc.all_reduce(a))
    if rank == 0:
        print(f"{label}: gemm+res {t_g:.3f} ms | gemm+nccl AR {t_n:.3f} | fused gemm-AR {t_f:.3f} | nccl AR alone {t_ar_n:.3f} | peer AR alone {t_ar_p:.3f}")
for (Nout, K, label) in [(6144, 4096, "qkv dgrad"), (11008, 4096, "gate/up dgrad")]:
    dy = torch.randn(M, Nout, device=dev).to(torch.bfloat16); w = (torch.randn(Nout, K, device=dev) * 0.02).to(torch.bfloat16)
    t_g = tm(lambda: gemm.mm_nn(dy, w))
    def nccl_d():
        y = gemm.mm_nn(dy, w); dist.all_reduce(y); return y
    t_n = tm(nccl_d)
    t_f = tm(lambda: tpc.gemm_all_reduce_dgrad(dy, w))
    if rank == 0:
        print(f"{label}: dgrad {t_g:.3f} ms | dgrad+nccl AR {t_n:.3f} | fused dgrad-AR {t_f:.3f}")
symmetric.release_all(); dist.barrier(); dist.destroy_process_group()
