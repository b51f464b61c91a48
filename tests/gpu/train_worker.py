"""torchrun worker: bit-exact resume and activation checkpointing on the GPU path.

Run by ``test_train_gpu.py`` with 1 rank (tp=1), 2 ranks (tp=2) or 4 ranks
(tp=2 x dp=2, the 2-D layout with ZeRO sharded checkpoints; ``DTB_TEST_TP``).  A
continuous run and a save-at-step-3 / resume run must give identical losses
and fp32 master weights, and a run with per-block activation checkpointing
must match the run without it bit for bit.  Prints TRAIN_OK on success.
"""
import os
import sys
import tempfile

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from build_your_own_distributed_training_b200.checkpointing.checkpoint import load_checkpoint, save_checkpoint  # noqa: E402
from build_your_own_distributed_training_b200.ops._ext import native  # noqa: E402
from build_your_own_distributed_training_b200.parallel.process_groups import build_process_context  # noqa: E402
from build_your_own_distributed_training_b200.training.loop import train_step  # noqa: E402
from build_your_own_distributed_training_b200.training.trainer import Trainer  # noqa: E402
from tests.helpers import tiny_config  # noqa: E402


def config(tmp, tp, ac=False):
    return tiny_config(tmp, run_id="gpu_resume", backend="nccl",
                       model__vocab_size=512, model__d_model=256, model__n_layers=2, model__n_heads=4,
                       model__n_kv_heads=2, model__ffn_hidden_size=512, model__max_seq_len=128,
                       data__seq_len=128, data__micro_batch_size=2, data__global_batch_size=0,
                       data__dataset_path="uniform", grad_accum_steps=1,
                       parallel__tp_size=tp, parallel__param_dtype="bfloat16",
                       parallel__activation_checkpointing=ac)


def steps(t, ctx, cfg, n):
    out = []
    for _ in range(n):
        w, _ = t._next_window()
        out.append(train_step(t.model, w, t.optimizer, t.scheduler, ctx, cfg, gpu_type="b200").loss)
        t.step += 1
    return out


def main():
    tp = int(os.environ.get("DTB_TEST_TP", os.environ["WORLD_SIZE"]))
    ctx = build_process_context(tp, backend="nccl", verbose=False)
    tmp = tempfile.mkdtemp() if ctx.rank == 0 else None
    box = [tmp]
    dist.broadcast_object_list(box, src=0)
    tmp = box[0]

    cfg = config(tmp, tp)
    a = Trainer(cfg, ctx=ctx, gpu_type="b200")
    la = steps(a, ctx, cfg, 3)
    path = save_checkpoint(a.model, a.optimizer, a.scheduler, a.step, cfg, ctx)
    la += steps(a, ctx, cfg, 3)
    wa = [u.master.clone() for u in a.model.units]

    b = Trainer(cfg, ctx=ctx, gpu_type="b200")
    b.step = load_checkpoint(b.model, b.optimizer, b.scheduler, path, ctx)
    b._fast_forward_data(b.step)
    lb = steps(b, ctx, cfg, 3)
    assert lb == la[3:], ("resume differs", la, lb)
    for x, y in zip(wa, [u.master for u in b.model.units]):
        assert torch.equal(x, y), "resumed weights differ"

    cfg_ac = config(tmp, tp, ac=True)
    c = Trainer(cfg_ac, ctx=ctx, gpu_type="b200")
    lc = steps(c, ctx, cfg_ac, 3)
    assert lc == la[:3], ("activation checkpointing changed the loss", la[:3], lc)
    assert native().device_error() == 0
    del a, b, c
    torch.cuda.synchronize()
    dist.barrier()
    if ctx.rank == 0:
        print("TRAIN_OK", la, flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
