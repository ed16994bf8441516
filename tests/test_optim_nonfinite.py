"""A non-finite gradient norm skips the AdamW update (parameters, moments and the step's bias
correction stay as they were) and stops training at the next log point, like a NaN loss.
CPU path here; the device path (NaN clip coefficient read by the AdamW kernel) has a GPU test."""
import math

import pytest
import torch

from oxidizr_b200.optim import AdamW, AdamWConfig, FlatParams


def _opt(device="cpu"):
    torch.manual_seed(0)
    ps = [torch.nn.Parameter(torch.randn(37, device=device)), torch.nn.Parameter(torch.randn(5, 8, device=device))]
    return ps, AdamW(FlatParams([("a", ps[0]), ("b", ps[1])], torch.device(device)), AdamWConfig(lr=1e-2))


def _state(opt):
    return [t.clone() for t in (opt.flat.master, opt.m, opt.v, opt.flat.flat)]


@pytest.mark.parametrize("bad", [float("inf"), float("nan")])
def test_nonfinite_gradient_skips_the_update(bad):
    ps, opt = _opt()
    ps[0].main_grad.fill_(0.1)
    ps[1].main_grad.fill_(-0.2)
    opt.step()
    before = _state(opt)
    ps[0].main_grad.fill_(0.1)
    ps[1].main_grad[2, 3] = bad
    nrm = float(opt.step())
    assert not math.isfinite(nrm)
    assert all(torch.equal(x, y) for x, y in zip(before, _state(opt)))
    assert float(opt.flat.grad.abs().sum()) == 0.0  # gradients were consumed (zeroed)
    # the next finite step updates again
    ps[0].main_grad.fill_(0.1)
    assert math.isfinite(float(opt.step()))
    assert not torch.equal(before[0], opt.flat.master)


def test_trainer_stops_on_nonfinite_grad_norm():
    from oxidizr_b200.trainer import NonFiniteLoss, Trainer
    t = Trainer.__new__(Trainer)
    t._check_finite(2.5, 1.0)
    with pytest.raises(NonFiniteLoss, match="gradient norm"):
        t._check_finite(2.5, float("inf"))
    with pytest.raises(NonFiniteLoss, match="NaN loss"):
        t._check_finite(float("nan"), 1.0)


@pytest.mark.gpu
def test_nonfinite_gradient_skips_the_update_on_device():
    ps, opt = _opt("cuda")
    ps[0].main_grad.fill_(0.1)
    ps[1].main_grad.fill_(-0.2)
    opt.step()
    before = _state(opt)
    st_before = opt._step_state.clone()
    ps[0].main_grad.fill_(0.1)
    ps[1].main_grad[2, 3] = float("inf")
    nrm = float(opt.step())
    torch.cuda.synchronize()
    assert not math.isfinite(nrm)
    assert all(torch.equal(x, y) for x, y in zip(before, _state(opt)))
    assert torch.equal(st_before, opt._step_state)  # bias-correction step not advanced
    ps[0].main_grad.fill_(0.1)
    assert math.isfinite(float(opt.step()))
    assert not torch.equal(before[0], opt.flat.master)
