"""Bit-exact resume and activation-checkpointing equality on the GPU path (1, 2 and 4 GPUs)."""

import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a GPU", allow_module_level=True)

HERE = os.path.dirname(os.path.abspath(__file__))


def _failure_text(r) -> str:
    """The ranks' exception lines first (torchrun's summary hides them), then the output tails."""
    errs = [ln for ln in r.stderr.splitlines() if "Error" in ln or "error:" in ln][:40]
    return "\n".join(errs) + "\n---\n" + r.stdout[-2000:] + r.stderr[-2000:]


@pytest.mark.parametrize("n,tp", [(1, 1), (2, 2), (4, 2)])
def test_resume_and_checkpointing_are_bit_exact(n, tp):
    if torch.cuda.device_count() < n:
        pytest.skip(f"needs {n} GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", DTB_PG_TIMEOUT_S="120", DTB_TEST_TP=str(tp))
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={n}",
           "--master-addr", "127.0.0.1", "--master-port", str(29681 + n), os.path.join(HERE, "train_worker.py")]
    r = subprocess.run(["timeout", "-k", "30", "600"] + cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0 and "TRAIN_OK" in r.stdout, _failure_text(r)
