"""Projection GEMM parity on the GPU (kf_linear_fwd through the C ABI and projection.linear).

Oracle: ``oracle.sana.linear_exact``, float64 ``x @ W^T + b`` (the nn.Linear layers of
LiteLA.forward, SANA_LinearAttention/original.py:122, 143; the reference's TileLang GEMMs of
custom.py:23-85, 457-523 accumulate in fp32 and round once, as this kernel does).
Bar: 16-bit outputs within 1 ulp + atol 1e-3 of the float64 value (inside the stated 1 ulp +
1e-2); fp32 outputs rtol 1e-4. Both weight layouts (nn.Linear [out, in] and the reference's
prepacked WeightT [in, out]), with and without a bias, tails in every dimension, and the
BASELINE SANA shapes (rows sampled at full size).
"""

import pytest
import torch

from oracle.sana import linear_exact
from tests.tolerances import assert_close_ulp_atol

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def proj():
    if not torch.cuda.is_available():
        pytest.skip("CUDA is required")
    from kernelforge_b200.SANA_LinearAttention import projection

    return projection


def _inputs(m, k, n, dtype, seed, bias=True):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=g).to(dtype)
    w = (torch.randn(n, k, generator=g) / k ** 0.5).to(dtype)
    b = torch.randn(n, generator=g).to(dtype) if bias else None
    return x, w, b


def _check(actual, expected, dtype):
    if dtype == torch.float32:
        torch.testing.assert_close(actual.cpu().double(), expected, rtol=1e-4, atol=1e-5)
    else:
        assert_close_ulp_atol(actual, expected, dtype=dtype, ulps=1, atol=1e-3)


SHAPES = [
    (1000, 1152, 3456),   # SANA-600M QKV projection (C = 1152), rows not a multiple of 128
    (515, 1152, 1152),    # its output projection
    (300, 2240, 6720),    # SANA-1600M QKV projection (C = 2240)
    (257, 2240, 2240),    # its output projection
    (7, 40, 24),          # K below one 64-wide stage, N below one 32-column chunk
    (129, 72, 200),       # K and N tails
    (384, 256, 512),      # exact tiles, several per CTA
]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", SHAPES)
def test_linear_against_float64(proj, shape, dtype):
    m, k, n = shape
    x, w, b = _inputs(m, k, n, dtype, seed=m + k + n)
    expected = linear_exact(x, w, b)
    dev = [t.cuda() for t in (x, w, b)]
    _check(proj.linear(*dev), expected, dtype)
    # The reference's prepacked WeightT [in, out] layout, and no bias.
    _check(proj.linear_t(dev[0], dev[1].t().contiguous(), dev[2]), expected, dtype)
    _check(proj.linear(dev[0], dev[1]), linear_exact(x, w), dtype)


@pytest.mark.parametrize("layout", ["nk", "kn"])
def test_linear_fp32(proj, layout):
    x, w, b = _inputs(100, 96, 80, torch.float32, seed=3)
    xd, wd, bd = x.cuda(), w.cuda(), b.cuda()
    y = proj.linear(xd, wd, bd) if layout == "nk" else proj.linear_t(xd, wd.t().contiguous(), bd)
    _check(y, linear_exact(x, w, b), torch.float32)


@pytest.mark.parametrize("cfg", [(4, 4096, 1152), (2, 16384, 2240)])
def test_baseline_projection_shapes(proj, cfg):
    """The two SANA BASELINE configurations' projections at full size: x [B*N, C] -> packed qkv
    [B*N, 3C] and the bias-fused output projection; 512 sampled rows against float64, the whole
    output deterministic across calls."""
    batch, seq, c = cfg
    m = batch * seq
    g = torch.Generator(device="cuda").manual_seed(c)
    x = torch.randn(m, c, device="cuda", generator=g).to(torch.bfloat16)
    wqkv = (torch.randn(3 * c, c, device="cuda", generator=g) / c ** 0.5).to(torch.bfloat16)
    wo = (torch.randn(c, c, device="cuda", generator=g) / c ** 0.5).to(torch.bfloat16)
    bo = torch.randn(c, device="cuda", generator=g).to(torch.bfloat16)
    qkv = proj.linear(x, wqkv)
    out = proj.linear(x, wo, bo)
    assert torch.equal(proj.linear(x, wqkv), qkv)
    rows = torch.randint(0, m, (512,), generator=torch.Generator().manual_seed(0)).cuda()
    _check(qkv[rows], linear_exact(x[rows], wqkv), torch.bfloat16)
    _check(out[rows], linear_exact(x[rows], wo, bo), torch.bfloat16)


def test_strided_weight_views_and_batched_input(proj):
    """A transposed view of either layout is read in place; [B, N, C] inputs keep their shape."""
    x, w, b = _inputs(2 * 33, 128, 96, torch.bfloat16, seed=11)
    xd = x.cuda().view(2, 33, 128)
    wd, bd = w.cuda(), b.cuda()
    expected = linear_exact(x, w, b).view(2, 33, 96)
    y1 = proj.linear(xd, wd, bd)
    y2 = proj.linear(xd, wd.t().contiguous().t(), bd)  # [out, in] view of a dense [in, out]
    y3 = proj.linear_t(xd, wd.t(), bd)                  # [in, out] view of a dense [out, in]
    for y in (y1, y2, y3):
        assert y.shape == (2, 33, 96)
        _check(y, expected, torch.bfloat16)
    assert torch.equal(y1, y3)


def test_empty_rows_and_errors(proj):
    from kernelforge_b200 import _lib

    w = torch.zeros(16, 8, dtype=torch.bfloat16, device="cuda")
    y = proj.linear(torch.zeros(0, 8, dtype=torch.bfloat16, device="cuda"), w)
    assert y.shape == (0, 16)
    with pytest.raises(RuntimeError, match="unsupported"):  # 16-bit out_features not a multiple of 8
        proj.linear(torch.zeros(4, 8, dtype=torch.bfloat16, device="cuda"),
                    torch.zeros(12, 8, dtype=torch.bfloat16, device="cuda"))
    with pytest.raises(ValueError):
        proj.linear(torch.zeros(4, 9, dtype=torch.bfloat16, device="cuda"), w)
    assert _lib.query_device_error() == 0
