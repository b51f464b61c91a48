"""Flash-attention throughput: tcgen05 forward/backward vs the mma.sync kernels and torch SDPA.

    python tests/performance/bench_attention.py
"""
import os, sys, math
sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
import torch
import torch.nn.functional as F
from build_your_own_distributed_training_b200.ops._ext import native
def tm(f, it=10):
    for _ in range(3): f()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(it): f()
    e1.record(); torch.cuda.synchronize()
    return e0.elapsed_time(e1) / it / 1e3
for (b, s, nq, nkv, hd) in [(1, 4096, 32, 32, 128), (2, 4096, 16, 16, 128), (1, 8192, 4, 1, 128), (8, 2048, 6, 2, 64)]:
    qkv = torch.randn(b * s, (nq + 2 * nkv) * hd, device="cuda", dtype=torch.bfloat16)
    fl = 4 * b * nq * s * s * hd / 2
    t_tc = tm(lambda: native().attn_fwd(qkv, b, s, nq, nkv, hd, 1 / math.sqrt(hd)))
    t_lg = tm(lambda: native().attn_fwd(qkv, b, s, nq, nkv, hd, 1 / math.sqrt(hd), legacy=True))
    q = qkv[:, :nq * hd].view(b, s, nq, hd).transpose(1, 2).contiguous()
    k = qkv[:, nq * hd:(nq + nkv) * hd].view(b, s, nkv, hd).transpose(1, 2).repeat_interleave(nq // nkv, 1).contiguous()
    v = qkv[:, (nq + nkv) * hd:].view(b, s, nkv, hd).transpose(1, 2).repeat_interleave(nq // nkv, 1).contiguous()
    t_sd = tm(lambda: F.scaled_dot_product_attention(q, k, v, is_causal=True))
    qr, kr, vr = (x.detach().requires_grad_() for x in (q, k, v))
    out = F.scaled_dot_product_attention(qr, kr, vr, is_causal=True)
    go = torch.randn_like(out)
    t_sdb = tm(lambda: torch.autograd.grad(out, (qr, kr, vr), go, retain_graph=True))
    o, lse = native().attn_fwd(qkv, b, s, nq, nkv, hd, 1 / math.sqrt(hd))
    do = torch.randn_like(o)
    t_myb = tm(lambda: native().attn_bwd(do, qkv, o, lse, b, s, nq, nkv, hd, 1 / math.sqrt(hd)))
    print(f"b{b} s{s} h{nq}/{nkv} hd{hd}: fwd tc {fl/t_tc/1e12:6.0f} TF/s | fwd mma.sync {fl/t_lg/1e12:6.0f} | "
          f"torch sdpa fwd {fl/t_sd/1e12:6.0f} | bwd mine {2.5*fl/t_myb/1e12:6.0f} | sdpa bwd {2.5*fl/t_sdb/1e12:6.0f}")
with torch.backends.cuda.sdp_kernel(enable_flash=False, enable_math=False, enable_mem_efficient=False, enable_cudnn=True) if hasattr(torch.backends.cuda, "sdp_kernel") else torch.no_grad():
    pass
print("sdpa backends:", torch.backends.cuda.flash_sdp_enabled(), torch.backends.cuda.cudnn_sdp_enabled(), torch.backends.cuda.mem_efficient_sdp_enabled())
