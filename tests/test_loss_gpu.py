"""hx_l2_loss_grad (gsplat.loss.l2_loss_grad) against a plain PyTorch fp32
reference: the mean-squared error and its gradient, on the 16-byte-aligned
vector path and the scalar path, ragged lengths, accumulation into a given
loss and a caller-chosen normaliser."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def _ref(p, t, inv_n):
    d = p.double() - t.double()
    return float((d * d).sum() * inv_n), (d * (2.0 * inv_n)).float()


@pytest.mark.parametrize("n", [1, 3, 4, 1000, 1023, 3 * 1080 * 1920, 5_000_001])
@pytest.mark.parametrize("offset", [0, 1])
def test_l2_loss_grad_matches_torch(n, offset):
    from gsplat.loss import l2_loss_grad

    g = torch.Generator().manual_seed(n + offset)
    base_p = torch.rand(n + offset, generator=g).cuda()
    base_t = torch.rand(n + offset, generator=g).cuda()
    p, t = base_p[offset:], base_t[offset:]  # offset 1: not 16-byte aligned (scalar path)
    loss, grad = l2_loss_grad(p, t)
    want_loss, want_grad = _ref(p, t, 1.0 / n)
    assert grad.shape == p.shape
    torch.testing.assert_close(grad, want_grad.cuda(), rtol=1e-6, atol=1e-12)
    assert abs(float(loss) - want_loss) <= 1e-5 * abs(want_loss) + 1e-7


def test_l2_loss_grad_accumulates_and_scales():
    from gsplat.loss import l2_loss_grad

    g = torch.Generator().manual_seed(3)
    p = torch.rand((3, 64, 96), generator=g).cuda()
    t = torch.rand((3, 64, 96), generator=g).cuda()
    acc = torch.full((1,), 0.25, device="cuda")
    out = torch.empty_like(p)
    loss, grad = l2_loss_grad(p, t, inv_n=1.0 / 7.0, loss=acc, grad=out)
    assert loss is acc and grad is out
    want_loss, want_grad = _ref(p, t, 1.0 / 7.0)
    torch.testing.assert_close(grad, want_grad.cuda(), rtol=1e-6, atol=1e-12)
    assert abs(float(acc) - (0.25 + want_loss)) <= 1e-5 * (0.25 + want_loss)


def test_l2_loss_grad_empty_and_errors():
    from gsplat.loss import l2_loss_grad

    e = torch.empty(0, device="cuda")
    loss, grad = l2_loss_grad(e, e)
    assert float(loss) == 0.0 and grad.numel() == 0
    with pytest.raises(RuntimeError):
        l2_loss_grad(torch.zeros(4, device="cuda"), torch.zeros(5, device="cuda"))
    with pytest.raises(RuntimeError):
        l2_loss_grad(torch.zeros(4, device="cuda", dtype=torch.float64),
                     torch.zeros(4, device="cuda", dtype=torch.float64))


def test_mse_loss_autograd():
    from gsplat.loss import mse_loss

    g = torch.Generator().manual_seed(11)
    p = torch.rand((3, 40, 56), generator=g).cuda().requires_grad_()
    t = torch.rand((3, 40, 56), generator=g).cuda()
    loss = mse_loss(p * 1.5, t)
    loss.backward()
    q = p.detach().clone().requires_grad_()
    want = ((q * 1.5 - t) ** 2).mean()
    want.backward()
    assert loss.shape == () and abs(float(loss) - float(want)) <= 1e-5 * float(want)
    torch.testing.assert_close(p.grad, q.grad, rtol=1e-5, atol=1e-9)
