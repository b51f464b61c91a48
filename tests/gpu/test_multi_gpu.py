"""NVLink transport on 2+ GPUs (skipped on a single-GPU box) and the timeout path on one GPU."""

import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a GPU", allow_module_level=True)

from build_your_own_distributed_training_b200.ops._ext import native  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))


def test_bounded_wait_times_out_and_reports():
    """A wait on a flag nothing sets returns after its limit with an error status."""
    native().device_error()  # clear
    flag = torch.zeros(4, dtype=torch.int32, device="cuda")
    native().wait_flag_probe(flag, 1, 0.05)
    assert native().device_error() == 2  # ERR_PEER_TIMEOUT
    # the context is still usable
    assert float(torch.ones(3, device="cuda").sum()) == 3.0



def _failure_text(r) -> str:
    """The ranks' exception lines first (torchrun's summary hides them), then the output tails."""
    errs = [ln for ln in r.stderr.splitlines() if "Error" in ln or "error:" in ln][:40]
    return "\n".join(errs) + "\n---\n" + r.stdout[-2000:] + r.stderr[-2000:]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_peer_collectives_and_fused_gemm_allreduce_match_nccl():
    n = min(torch.cuda.device_count(), 8)
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={n}",
           "--master-addr", "127.0.0.1", "--master-port", "29671", os.path.join(HERE, "mgpu_worker.py")]
    r = subprocess.run(["timeout", "-k", "30", "600"] + cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0 and "MGPU_OK" in r.stdout, _failure_text(r)
