"""CPU oracle for the RMSNorm forward -- TEST INFRASTRUCTURE ONLY (see ``oracle/__init__``).

Restates ``RMSNorm._norm`` / ``RMSNorm.forward`` of the reference
(rmsnorm/original.py:27-38 and :40-52):

    y = cast_to_input_dtype( x_f32 * rsqrt(mean(x_f32 ** 2) + eps) ) * weight

The normalised row is rounded to the input dtype *before* the weight multiply, and the
weight multiply rounds again (the reference's ``.type_as(x)`` followed by ``* self.weight``;
the one-pass kernel of rmsnorm/custom.py:63-73 keeps the same double rounding).
"""

from __future__ import annotations

import torch


def rmsnorm_forward(x: torch.Tensor, weight: torch.Tensor | None, eps: float = 1e-6) -> torch.Tensor:
    """Reference-semantics RMSNorm on the CPU (fp32 statistics, double rounding).

    ``weight=None`` gives the normalised row only (the "original TileLang" comparator of
    rmsnorm/original.py:55-78 has no weight).
    """
    xf = x.detach().to("cpu", torch.float32)
    dim = xf.shape[-1]
    mean_sq = (xf * xf).sum(dim=-1, keepdim=True) / dim
    scale = 1.0 / torch.sqrt(mean_sq + eps)
    normed = (xf * scale).to(x.dtype)
    if weight is None:
        return normed
    # Same-dtype multiply: torch evaluates bf16/fp16 products in fp32 and rounds once.
    return normed * weight.detach().to("cpu")


def rmsnorm_exact(x: torch.Tensor, weight: torch.Tensor | None, eps: float = 1e-6) -> torch.Tensor:
    """Float64 statistics with the reference's rounding points, for tight GPU checks."""
    xd = x.detach().to("cpu", torch.float64)
    dim = xd.shape[-1]
    scale = 1.0 / torch.sqrt((xd * xd).sum(dim=-1, keepdim=True) / dim + eps)
    normed = (xd * scale).to(x.dtype)
    if weight is None:
        return normed
    return (normed.double() * weight.detach().to("cpu", torch.float64)).to(x.dtype)


def rmsnorm_backward(x: torch.Tensor, weight: torch.Tensor | None, dy: torch.Tensor, eps: float = 1e-6):
    """Float64 gradients (dx, dweight) of the reference forward (rmsnorm/original.py:40-52).

    The reference has no backward (rmsnorm/README.md:5); this differentiates its forward
    ``y = (x * rsqrt(mean(x^2) + eps)).type_as(x) * weight`` with torch autograd, the casts
    taken as identities as autograd does, while the weight gradient sees the rounded
    normalised row ``(x * r).type_as(x)`` the forward multiplies by. ``dweight`` is None when
    ``weight`` is None.
    """
    xd = x.detach().to("cpu", torch.float64).requires_grad_()
    dim = xd.shape[-1]
    scale = 1.0 / torch.sqrt((xd * xd).sum(dim=-1, keepdim=True) / dim + eps)
    normed = xd * scale
    dyd = dy.detach().to("cpu", torch.float64)
    if weight is None:
        (dx,) = torch.autograd.grad(normed, (xd,), dyd)
        return dx, None
    wd = weight.detach().to("cpu", torch.float64).requires_grad_()
    (dx,) = torch.autograd.grad(normed * wd, (xd,), dyd)
    rounded = (x.detach().to("cpu", torch.float64) * scale.detach()).to(x.dtype).double()
    dw = (dyd * rounded).reshape(-1, dim).sum(0)
    return dx, dw
