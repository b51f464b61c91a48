"""The allocation-free RMSNorm backward, called through its exported C symbol.

It serves callers that cannot allocate device memory when they run the
backward (a host program linking the library without PyTorch's allocator, or
one whose device memory is all reserved up front).  Its results must match
the allocating entry point's.  This file (in the last directory of tests/) is
collected last so a run that stops at the first failure has run every other
test first.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a GPU", allow_module_level=True)

from build_your_own_distributed_training_b200.ops._ext import native  # noqa: E402

DEV = torch.device("cuda", 0)


def _entry():
    lib = ctypes.CDLL(native().__file__)
    fn = lib.dtb_rmsnorm_bwd_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p,
                   ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    err = lib.dtb_noalloc_error_string
    err.restype = ctypes.c_char_p
    err.argtypes = [ctypes.c_int]
    return fn, err


def _rel(a, b):
    a, b = a.float(), b.float()
    return float((a - b).norm() / b.norm().clamp_min(1e-12))


@pytest.mark.parametrize("w_dtype", [torch.bfloat16, torch.float32])
def test_noalloc_matches_allocating_entry_point_on_two_calls(w_dtype):
    fn, err = _entry()
    torch.manual_seed(0)
    stream = torch.cuda.current_stream(DEV)
    for rows, dim in ((3000, 4096), (513, 2048)):  # two calls in a row, different sizes
        x = torch.randn(rows, dim, device=DEV).to(torch.bfloat16)
        dy = torch.randn(rows, dim, device=DEV).to(torch.bfloat16)
        w = (1 + 0.1 * torch.randn(dim, device=DEV)).to(w_dtype)
        _, rstd = native().rmsnorm_fwd(x, w, 1e-5)
        acc_ref = torch.full((dim,), 0.5, device=DEV)
        dx_ref = native().rmsnorm_bwd(dy, x, w, rstd, acc_ref)
        dx = torch.empty_like(x)
        acc = torch.full((dim,), 0.5, device=DEV)
        torch.cuda.synchronize()
        rc = fn(dy.data_ptr(), x.data_ptr(), w.data_ptr(), int(w_dtype == torch.float32), rstd.data_ptr(),
                dx.data_ptr(), acc.data_ptr(), rows, dim, ctypes.c_void_p(stream.cuda_stream))
        assert rc == 0, err(rc).decode()
        torch.cuda.synchronize()
        assert _rel(dx, dx_ref) < 2e-2
        assert torch.equal(dx, dx_ref)  # same per-row arithmetic
        assert _rel(acc - 0.5, acc_ref - 0.5) < 1e-5  # partial sums taken in another grouping


def test_noalloc_rejects_sizes_beyond_the_limit():
    fn, err = _entry()
    t = torch.zeros(8, 16384, device=DEV, dtype=torch.bfloat16)
    r = torch.ones(8, device=DEV)
    acc = torch.zeros(16384, device=DEV)
    rc = fn(t.data_ptr(), t.data_ptr(), acc.data_ptr(), 1, r.data_ptr(), t.data_ptr(), acc.data_ptr(), 8, 16384,
            None)
    assert rc == 2 and b"12288" in err(rc)
    rc = fn(t.data_ptr(), t.data_ptr(), acc.data_ptr(), 1, r.data_ptr(), t.data_ptr(), acc.data_ptr(), 8, 100, None)
    assert rc == 1


def test_noalloc_rejects_misaligned_pointers_without_launching():
    fn, err = _entry()
    t = torch.zeros(8 * 64 + 8, device=DEV, dtype=torch.bfloat16)
    x = t[1:1 + 8 * 64]  # 2 bytes past a 16-byte boundary
    r = torch.ones(8, device=DEV)
    acc = torch.zeros(64, device=DEV)
    w = torch.ones(64, device=DEV)
    rc = fn(x.data_ptr(), x.data_ptr(), w.data_ptr(), 1, r.data_ptr(), x.data_ptr(), acc.data_ptr(), 8, 64, None)
    assert rc == 1 and b"16-byte" in err(rc)
    torch.cuda.synchronize()
    assert torch.count_nonzero(acc) == 0  # nothing ran
