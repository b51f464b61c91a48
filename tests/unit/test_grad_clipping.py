import pytest
import torch

from build_your_own_distributed_training_b200.training.grad_utils import (GradNotFiniteError, clip_grad_norm_,
                                                                          device_clip_state, grad_finite_check)


def _params(*grads):
    ps = []
    for g in grads:
        p = torch.nn.Parameter(torch.zeros_like(g))
        p.grad = g.clone()
        ps.append(p)
    return ps


def test_norm_and_clip():
    ps = _params(torch.full((4,), 3.0), torch.full((3,), 4.0))
    total = (4 * 9 + 3 * 16) ** 0.5
    assert abs(clip_grad_norm_(ps, 1.0) - total) < 1e-5
    now = torch.sqrt(sum(p.grad.pow(2).sum() for p in ps))
    assert abs(float(now) - 1.0) < 1e-4


def test_no_clip_below_threshold_and_disabled():
    ps = _params(torch.full((2,), 0.1))
    clip_grad_norm_(ps, 10.0)
    assert torch.allclose(ps[0].grad, torch.full((2,), 0.1))
    n = clip_grad_norm_(_params(torch.full((2,), 100.0)), 0.0)
    assert abs(n - 200 ** 0.5 * 10) < 1e-3


def test_device_clip_state():
    s = device_clip_state(torch.tensor(4.0), 1.0)
    assert abs(float(s[0]) - 1 / (4 + 1e-6)) < 1e-7 and float(s[1]) == 1.0
    s = device_clip_state(torch.tensor(float("nan")), 1.0)
    assert float(s[1]) == 0.0
    assert float(device_clip_state(torch.tensor(0.5), 1.0)[0]) == 1.0


@pytest.mark.parametrize("bad", [float("nan"), float("inf")])
def test_finite_check_raises(single_process_pg, bad):
    ps = _params(torch.tensor([1.0, bad]))
    with pytest.raises(GradNotFiniteError):
        grad_finite_check(ps)
    assert grad_finite_check(_params(torch.ones(3)))
