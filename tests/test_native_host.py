"""Host-side behaviour of the native extension that needs no GPU."""
import pytest

from oxidizr_b200.ops._C import raw_ext


def test_failed_launcher_check_raises_python_error():
    e = raw_ext()
    e.host_check_selftest(0)
    with pytest.raises(RuntimeError, match="value 3 of 2.5 true"):
        e.host_check_selftest(3)


def test_split_cols_gradient_matches_slicing():
    import torch
    from oxidizr_b200.ops.api import split_cols
    p = torch.randn(2, 3, 10, requires_grad=True)
    a, b, c = split_cols(p, [4, 5, 1])
    (a.sum() * 2 + (b ** 2).sum()).backward()  # c unused: zero gradient block
    q = p.detach().clone().requires_grad_()
    (q[..., :4].sum() * 2 + (q[..., 4:9] ** 2).sum()).backward()
    assert torch.equal(p.grad, q.grad)
