"""Lazily zeroed gradient slices: take / zero-on-overlap / flush semantics."""
import torch

from build_your_own_distributed_training_b200.ops import gemm, grad_state


def _fresh(n=64):
    buf = torch.full((n,), 7.0)           # stale contents from an earlier step
    fs = grad_state.FreshSet(buf)
    fs.mark([(0, 16), (16, 16), (32, 16), (48, 16)])
    return buf, fs


def test_take_exact_run_then_not_fresh():
    buf, fs = _fresh()
    assert fs.take(0, 16)                 # one range
    assert not fs.take(0, 16)             # already written this step
    assert fs.take(16, 32)                # a stacked view over two adjacent ranges
    assert set(fs.ranges) == {48}


def test_partial_overlap_zeroes_the_fresh_part():
    buf, fs = _fresh()
    assert fs.take(0, 16)
    buf[0:16] = 1.0                       # the first writer stored its gradient
    # a view over [0, 32): half written, half fresh -> accumulate after zeroing the fresh half
    assert not fs.take(0, 32)
    assert torch.equal(buf[0:16], torch.ones(16)) and not buf[16:32].any()
    assert 16 not in fs.ranges


def test_flush_zeroes_unwritten_slices():
    buf, fs = _fresh()
    fs.take(32, 16)
    buf[32:48] = 3.0
    fs.flush()
    assert not buf[0:32].any() and not buf[48:].any()
    assert torch.equal(buf[32:48], torch.full((16,), 3.0))
    assert not fs.ranges


def test_tagged_views_store_then_accumulate():
    buf, fs = _fresh()
    view = grad_state.tag(buf[16:32].view(4, 4), fs, 16)
    a, b = torch.randn(8, 4), torch.randn(8, 4)
    gemm.mm_tn_into_grad(a, b, view, (4, 4))          # first write: overwrites the stale 7.0s
    torch.testing.assert_close(buf[16:32].view(4, 4), a.t() @ b)
    gemm.mm_tn_into_grad(a, b, view, (4, 4))          # second write: accumulates
    torch.testing.assert_close(buf[16:32].view(4, 4), 2 * (a.t() @ b))
    untagged = torch.ones(4, 4)
    assert not grad_state.take_fresh(untagged) and not grad_state.take_fresh(None)


def test_zero_if_fresh_for_accumulate_only_writers():
    buf, fs = _fresh()
    view = grad_state.tag(buf[48:64], fs, 48)
    grad_state.zero_if_fresh(view)
    assert not buf[48:64].any()
    buf[48:64] += 2.0
    grad_state.zero_if_fresh(view)        # no longer fresh: left alone
    assert torch.equal(buf[48:64], torch.full((16,), 2.0))
