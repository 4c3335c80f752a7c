"""Pin the CPU oracle against fixtures produced by running the reference itself (CPU only)."""

from pathlib import Path

import pytest
import torch

from oracle import fa_jvp, rmsnorm, sana
from tests.tolerances import assert_within_ulps

GOLDEN = Path(__file__).resolve().parent / "golden"


def _load(name):
    return torch.load(GOLDEN / name, weights_only=False)


@pytest.mark.parametrize("index", range(6))
def test_rmsnorm_oracle_matches_reference(index):
    case = _load("rmsnorm_golden.pt")[index]
    y = rmsnorm.rmsnorm_forward(case["x"], case["weight"], case["eps"])
    assert y.dtype == case["y"].dtype and y.shape == case["y"].shape
    exact = rmsnorm.rmsnorm_exact(case["x"], case["weight"], case["eps"])
    if y.dtype == torch.float32:
        # fp32 outputs: only the summation order differs (a few fp32 ulps).
        torch.testing.assert_close(y, case["y"], rtol=1e-5, atol=1e-6)
        torch.testing.assert_close(exact, case["y"], rtol=1e-5, atol=1e-6)
    else:
        # Same rounding points; only fp32 summation order differs -> at most one ulp, rarely.
        assert_within_ulps(y, case["y"], ulps=1)
        assert_within_ulps(exact, case["y"], ulps=1)


@pytest.mark.parametrize("index", range(6))
def test_sana_oracle_matches_reference(index):
    case = _load("sana_golden.pt")[index]
    qkv, heads, dim, eps = case["qkv"], case["heads"], case["dim"], case["eps"]
    ref = case["out"]
    mine = sana.qkv_attention_reference(qkv, heads, dim, eps)
    assert mine.dtype == torch.float32 and mine.shape == ref.shape
    torch.testing.assert_close(mine, ref, rtol=1e-6, atol=1e-6)
    # The float64 evaluation differs from the reference only by the reference's
    # intermediate low-precision roundings (vk and vk @ q are rounded to the input dtype).
    exact = sana.attn_exact(qkv, heads, dim, eps).float()
    tol = dict(rtol=1e-5, atol=1e-5) if qkv.dtype == torch.float32 else dict(rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(exact, ref, **tol)


@pytest.mark.parametrize("index", range(7))
def test_fa_oracle_matches_reference(index):
    case = _load("fa_jvp_golden.pt")[index]
    b, nq, nk, h, hk, d, causal, scale = case["case"]
    prim = [case[n].double() for n in ("q", "k", "v")]
    tang = [case[n].double() for n in ("tq", "tk", "tv")]
    out, tangent = fa_jvp.attention_jvp(*prim, *tang, softmax_scale=scale, causal=causal)
    torch.testing.assert_close(out.float(), case["out"], rtol=1e-6, atol=1e-6)
    torch.testing.assert_close(tangent.float(), case["tangent"], rtol=1e-6, atol=1e-6)
    lse = fa_jvp.attention_lse(*prim[:2], softmax_scale=scale, causal=causal).float()
    finite = torch.isfinite(case["lse"])
    assert torch.equal(finite, torch.isfinite(lse))
    torch.testing.assert_close(lse[finite], case["lse"][finite], rtol=1e-6, atol=1e-6)
    dense = fa_jvp.attention_jvp_from_forward(
        *(x.float() for x in prim), *(x.float() for x in tang), case["out"], case["lse"],
        softmax_scale=scale, causal=causal,
    )
    torch.testing.assert_close(dense, case["dense_from_forward"], rtol=1e-5, atol=1e-5)
    attn = fa_jvp.attention(*(x.float() for x in prim), softmax_scale=scale, causal=causal)
    torch.testing.assert_close(attn, case["attention_out_fp32"], rtol=1e-6, atol=1e-6)
    if causal and nq > nk:
        # Rows that see no key are exactly zero (flash_attention_jvp/test.py:83-84).
        assert torch.count_nonzero(tangent[:, : nq - nk]) == 0
        assert torch.isinf(lse[:, :, : nq - nk]).all()


def test_oracle_detects_a_planted_error():
    """A perturbed oracle must fail the golden check (the check is not vacuous)."""
    case = _load("rmsnorm_golden.pt")[0]
    wrong = rmsnorm.rmsnorm_forward(case["x"], case["weight"], case["eps"] * 1e4 + 1e-1)
    with pytest.raises(AssertionError):
        assert_within_ulps(wrong, case["y"], ulps=1)


@pytest.mark.parametrize("weighted", [True, False])
def test_rmsnorm_backward_oracle_matches_finite_differences(weighted):
    """The backward oracle (the reference has no RMSNorm backward) against central finite
    differences of the float64 forward y = x r w: dx exactly, dweight through the unrounded row
    (fp32 inputs, so the forward's cast is the identity)."""
    g = torch.Generator().manual_seed(5)
    x = torch.randn(3, 6, generator=g, dtype=torch.float64).float()
    w = (1 + 0.1 * torch.randn(6, generator=g, dtype=torch.float64)).float() if weighted else None
    dy = torch.randn(3, 6, generator=g, dtype=torch.float64).float()
    eps = 1e-6
    dx, dw = rmsnorm.rmsnorm_backward(x, w, dy, eps)

    def loss(xd, wd):
        r = 1.0 / torch.sqrt((xd * xd).mean(-1, keepdim=True) + eps)
        y = xd * r * (wd if wd is not None else 1.0)
        return (y * dy.double()).sum()

    xd, wd = x.double(), None if w is None else w.double()
    h = 1e-6
    num_dx = torch.zeros_like(xd)
    for i in range(xd.numel()):
        e = torch.zeros_like(xd).view(-1)
        e[i] = h
        e = e.view_as(xd)
        num_dx.view(-1)[i] = (loss(xd + e, wd) - loss(xd - e, wd)) / (2 * h)
    torch.testing.assert_close(dx, num_dx, rtol=1e-6, atol=1e-8)
    if weighted:
        num_dw = torch.zeros_like(wd)
        for i in range(wd.numel()):
            e = torch.zeros_like(wd)
            e[i] = h
            num_dw[i] = (loss(xd, wd + e) - loss(xd, wd - e)) / (2 * h)
        torch.testing.assert_close(dw, num_dw, rtol=1e-6, atol=1e-8)
    else:
        assert dw is None
