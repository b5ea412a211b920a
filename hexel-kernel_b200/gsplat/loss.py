"""Fit-step loss on the GPU in one pass (no reference counterpart: the
reference's training loops form the mean-squared error with torch ops)."""

from __future__ import annotations

from typing import Optional, Tuple

import torch

from ._lib import check_input, check_same_device, lib, ptr, stream


def l2_loss_grad(pred: torch.Tensor, target: torch.Tensor, *, inv_n: Optional[float] = None,
                 loss: Optional[torch.Tensor] = None,
                 grad: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """sum((pred - target)^2) * inv_n and its gradient 2 (pred - target) inv_n
    with respect to `pred`, in one kernel (hx_l2_loss_grad).  `inv_n`
    defaults to 1 / pred.numel() (the mean).  With `loss` (a one-element
    float32 CUDA tensor) the loss is ADDED to it; otherwise a new zeroed one
    receives it.  With `grad` the gradient is written there.  Returns
    (loss, grad)."""
    check_input(pred, "pred")
    check_input(target, "target")
    if pred.dtype != torch.float32 or target.dtype != torch.float32:
        raise RuntimeError("pred and target must be float32")
    if pred.shape != target.shape:
        raise RuntimeError(f"pred {tuple(pred.shape)} and target {tuple(target.shape)} differ")
    dev = pred.device
    if grad is None:
        grad = torch.empty_like(pred)
    else:
        check_input(grad, "grad")
        if grad.shape != pred.shape or grad.dtype != torch.float32:
            raise RuntimeError("grad must be float32 of pred's shape")
    if loss is None:
        loss = torch.zeros((1,), dtype=torch.float32, device=dev)
    elif not (loss.is_cuda and loss.dtype == torch.float32 and loss.numel() == 1):
        raise RuntimeError("loss must be a one-element float32 CUDA tensor")
    check_same_device(pred, "pred", target=target, grad=grad, loss=loss)
    n = pred.numel()
    scale = (1.0 / n if n else 0.0) if inv_n is None else float(inv_n)
    with torch.cuda.device(dev):
        lib.call("hx_l2_loss_grad", ptr(pred), ptr(target), n, scale, ptr(grad), ptr(loss),
                 stream(dev))
    return loss, grad


class _MSELoss(torch.autograd.Function):
    @staticmethod
    def forward(ctx, pred, target):
        loss, grad = l2_loss_grad(pred.contiguous(), target.contiguous())
        ctx.save_for_backward(grad)
        return loss.view(())

    @staticmethod
    def backward(ctx, g):
        (grad,) = ctx.saved_tensors
        return grad * g, None


def mse_loss(pred: torch.Tensor, target: torch.Tensor) -> torch.Tensor:
    """Differentiable mean((pred - target)^2) (gradient with respect to pred
    only) computed by l2_loss_grad: one kernel forms the loss and the
    gradient the backward returns."""
    return _MSELoss.apply(pred, target)
