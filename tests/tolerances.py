"""Tolerances shared by the parity tests.

The stated bars:
* integer / index work: bit-exact;
* bf16 / fp16 outputs: within 1 ulp of the oracle (``assert_within_ulps``), or, where the
  reference itself rounds intermediates differently from an fp32-accumulating kernel, within
  ``ulps`` ulp plus ``atol`` = 1e-2 (``assert_close_ulp_atol``);
* fp32 outputs: rtol 1e-4 (plus a small atol for values near zero).
"""

from __future__ import annotations

import torch

_MANTISSA_BITS = {torch.bfloat16: 7, torch.float16: 10, torch.float32: 23, torch.float64: 52}


def ulp_of(values: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """Spacing of ``dtype`` at |values| (normal range; subnormals use the smallest spacing)."""
    v = values.detach().to("cpu", torch.float64).abs()
    finfo = torch.finfo(dtype)
    exponent = torch.floor(torch.log2(torch.clamp_min(v, finfo.tiny)))
    return torch.pow(2.0, exponent - _MANTISSA_BITS[dtype])


def ulp_distance(actual: torch.Tensor, expected: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """Number of representable ``dtype`` values between actual and expected (both rounded to
    ``dtype``), from the ordering of their bit patterns."""
    int_type = {torch.bfloat16: torch.int16, torch.float16: torch.int16, torch.float32: torch.int32}[dtype]
    sign_mask = {torch.int16: 0x7FFF, torch.int32: 0x7FFFFFFF}[int_type]

    def key(t):
        i = t.detach().to("cpu").to(dtype).contiguous().view(int_type).to(torch.int64)
        return torch.where(i < 0, -(i & sign_mask), i)

    return (key(actual) - key(expected)).abs()


def assert_within_ulps(actual: torch.Tensor, expected: torch.Tensor, ulps: int = 1, dtype=None):
    dtype = dtype or expected.dtype
    assert actual.shape == expected.shape, (actual.shape, expected.shape)
    dist = ulp_distance(actual, expected, dtype)
    bad = dist > ulps
    if bad.any():
        a = actual.detach().to("cpu", torch.float64)
        e = expected.detach().to("cpu", torch.float64)
        idx = torch.nonzero(bad)[0].tolist()
        raise AssertionError(
            f"{int(bad.sum())} of {bad.numel()} elements differ by more than {ulps} ulp "
            f"(max {int(dist.max())}; first at {idx}: actual={a[tuple(idx)].item()!r} "
            f"expected={e[tuple(idx)].item()!r})"
        )


def assert_close_ulp_atol(actual, expected, *, dtype, ulps=1, atol=1e-2):
    """|actual - expected| <= atol + ulps * ulp_dtype(expected), elementwise."""
    a = actual.detach().to("cpu", torch.float64)
    e = expected.detach().to("cpu", torch.float64)
    assert a.shape == e.shape, (a.shape, e.shape)
    bound = atol + ulps * ulp_of(e, dtype)
    diff = (a - e).abs()
    bad = diff > bound
    if bad.any():
        idx = torch.nonzero(bad)[0].tolist()
        raise AssertionError(
            f"{int(bad.sum())} of {bad.numel()} elements outside atol={atol} + {ulps} ulp "
            f"(max diff {diff.max().item():.3g}; first at {idx}: "
            f"actual={a[tuple(idx)].item()!r} expected={e[tuple(idx)].item()!r})"
        )


def fa_tolerance(dtype):
    """FlashAttention-JVP tolerances of the reference harness (flash_attention_jvp/test.py:58-59)."""
    return {torch.float16: dict(atol=3e-3, rtol=1e-2), torch.bfloat16: dict(atol=3e-2, rtol=3e-2)}[dtype]


def assert_rmsnorm_close(actual, expected):
    """RMSNorm bar (rmsnorm/original.py:51-52 double rounding).

    The normalised row is rounded to the 16-bit dtype before the weight multiply. When the
    kernel's fp32 row scale differs from the oracle's in its last bit (summation order), the
    intermediate can round one ulp differently, and multiplying by a weight below one can turn
    that into two ulps of the output. So every element is within 2 ulps (ulp distance counted
    in representable values) and within the reference harness tolerance rtol = atol = 2e-2
    (rmsnorm/test.py:62-63). fp32 outputs: rtol 1e-5.
    """
    if expected.dtype == torch.float32:
        torch.testing.assert_close(actual.detach().cpu(), expected.detach().cpu(), rtol=1e-5, atol=1e-6)
        return
    assert_within_ulps(actual, expected, ulps=2)
    torch.testing.assert_close(actual.detach().cpu().float(), expected.detach().cpu().float(), rtol=2e-2, atol=2e-2)


def assert_rmsnorm_stated_bar(actual, normed, weight):
    """The stated bar for 16-bit RMSNorm outputs, 1 ulp + atol 1e-2 of the oracle, with the one
    exception that the reference's double rounding (rmsnorm/original.py:51-52) makes unavoidable.

    ``normed`` is the oracle's normalised row, already rounded to the dtype (the reference's
    ``.type_as(x)``), and ``weight`` the weight; the oracle's output is ``normed * weight``
    rounded once. An element outside the bar must equal the reference's second rounding applied
    to a neighbour (one ulp up or down) of ``normed``: the kernel's fp32 row scale differed from
    the oracle's in its last bits (summation order) and the normalised value rounded the other
    way. Anything else fails. Works on any device; returns the number of elements outside the
    bar (all of them explained).
    """
    dtype = normed.dtype
    expected = normed * weight
    a, e = actual.double(), expected.double()
    mag = e.abs().clamp_min(torch.finfo(dtype).tiny)
    ulp = torch.pow(2.0, torch.floor(torch.log2(mag)) - _MANTISSA_BITS[dtype])
    outside = (a - e).abs() > 1e-2 + ulp
    if not bool(outside.any()):
        return 0
    bits = normed.contiguous().view(torch.int16)
    neighbours = [(bits + step).view(dtype) * weight for step in (-1, 1)]
    explained = (actual == neighbours[0]) | (actual == neighbours[1])
    bad = outside & ~explained
    if bool(bad.any()):
        idx = torch.nonzero(bad)[0].tolist()
        raise AssertionError(
            f"{int(bad.sum())} of {bad.numel()} elements outside atol=1e-2 + 1 ulp and not explained by the "
            f"double rounding (first at {idx}: actual={a[tuple(idx)].item()!r} expected={e[tuple(idx)].item()!r})"
        )
    return int(outside.sum())
