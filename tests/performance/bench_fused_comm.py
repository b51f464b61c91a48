"""TP collectives on 2+ GPUs: fused GEMM+all-reduce (one-shot and two-shot) vs GEMM + NCCL
all-reduce, and the peer all-reduce vs NCCL, on 7B layer shapes split over the group.

    torchrun --nproc_per_node N tests/performance/bench_fused_comm.py

Times are CUDA events around 20 calls after 3 warm-ups, max over ranks.  ``roofline`` is the
slower of the GEMM at the measured bf16 peak and the bytes each rank must pull over NVLink
(770 GB/s per direction measured on this pool's B200s): (tp-1) payloads one-shot,
2(tp-1)/tp two-shot.
"""
import json
import os
import sys
from datetime import timedelta

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from build_your_own_distributed_training_b200.ops import gemm  # noqa: E402
from build_your_own_distributed_training_b200.parallel import symmetric  # noqa: E402

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
NVLINK_GBS = 770.0


def peak_tflops() -> float:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops"])
    except (OSError, KeyError, ValueError):
        return 1590.0


def main():
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    rank, world = dist.get_rank(), dist.get_world_size()
    dev = torch.device("cuda", local)

    def tm(f, it=20):
        for _ in range(3):
            f()
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(it):
            f()
        e1.record()
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) / it], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t)

    def roof(flops, payload_bytes, two_shot):
        pulls = (2 * (world - 1) / world if two_shot else (world - 1)) * payload_bytes
        return max(flops / (peak_tflops() * 1e12), pulls / (NVLINK_GBS * 1e9)) * 1e3

    M = 8192
    tpc = symmetric.TPComm(dist.group.WORLD, dev, M, 4096)
    for (K, N, label) in [(4096 // world, 4096, "wo fwd"), (11008 // world, 4096, "down fwd")]:
        x = torch.randn(M, K, device=dev).to(torch.bfloat16)
        w = (torch.randn(N, K, device=dev) * 0.02).to(torch.bfloat16)
        r = torch.randn(M, N, device=dev).to(torch.bfloat16)
        t_g = tm(lambda: gemm.mm_nt(x, w, residual=r))

        def nccl_path():
            y = gemm.mm_nt(x, w)
            dist.all_reduce(y)
            return y + r
        t_n = tm(nccl_path)
        res = {}
        for two in (False, True):
            tpc.two_shot = two
            res[two] = tm(lambda: tpc.gemm_all_reduce(x, w, r))
        a = torch.randn(M, N, device=dev).to(torch.bfloat16)
        t_ar_n = tm(lambda: dist.all_reduce(a))
        t_ar_p = tm(lambda: tpc.all_reduce(a))
        fl, pay = 2.0 * M * N * K, M * N * 2
        if rank == 0:
            print(f"tp={world} {label} M={M} N={N} K={K}: gemm+res {t_g:.3f} ms | gemm+NCCL AR {t_n:.3f} | "
                  f"fused one-shot {res[False]:.3f} (roofline {roof(fl, pay, False):.3f}) | "
                  f"fused two-shot {res[True]:.3f} (roofline {roof(fl, pay, True):.3f}) | "
                  f"NCCL AR alone {t_ar_n:.3f} | peer AR alone {t_ar_p:.3f}", flush=True)
    for (Nout, K, label) in [(3 * 4096 // world, 4096, "qkv dgrad"), (2 * 11008 // world, 4096, "gate/up dgrad")]:
        dy = torch.randn(M, Nout, device=dev).to(torch.bfloat16)
        w = (torch.randn(Nout, K, device=dev) * 0.02).to(torch.bfloat16)
        t_g = tm(lambda: gemm.mm_nn(dy, w))

        def nccl_d():
            y = gemm.mm_nn(dy, w)
            dist.all_reduce(y)
            return y
        t_n = tm(nccl_d)
        res = {}
        for two in (False, True):
            tpc.two_shot = two
            res[two] = tm(lambda: tpc.gemm_all_reduce_dgrad(dy, w))
        fl, pay = 2.0 * M * Nout * K, M * K * 2
        if rank == 0:
            print(f"tp={world} {label} M={M} N={K} K={Nout}: dgrad {t_g:.3f} ms | dgrad+NCCL AR {t_n:.3f} | "
                  f"fused one-shot {res[False]:.3f} (roofline {roof(fl, pay, False):.3f}) | "
                  f"fused two-shot {res[True]:.3f} (roofline {roof(fl, pay, True):.3f})", flush=True)
    symmetric.release_all()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
