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
