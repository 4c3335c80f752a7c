"""RMSNorm parity on the GPU: the CUDA kernel (through the C ABI) against the CPU oracle and the
reference-generated golden fixtures.

Bar (``tests.tolerances.assert_rmsnorm_close``): bf16/fp16 outputs within 2 ulps (the
reference's double rounding can turn a last-bit difference of the fp32 row scale into two
ulps of the output) and within the harness tolerance 2e-2; the weightless normalised row,
which is rounded once, within 1 ulp; fp32 outputs rtol 1e-5."""

from pathlib import Path

import pytest
import torch

from oracle import rmsnorm as oracle
from tests.tolerances import assert_rmsnorm_close, assert_rmsnorm_stated_bar, assert_within_ulps, ulp_distance

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def kf():
    if not torch.cuda.is_available():
        pytest.skip("CUDA is required")
    import kernelforge_b200.rmsnorm as mod

    return mod


def _check(actual, expected):
    assert_rmsnorm_close(actual, expected)


@pytest.mark.parametrize("index", range(6))
def test_golden_fixtures(kf, index):
    case = torch.load(GOLDEN / "rmsnorm_golden.pt", weights_only=False)[index]
    x, w = case["x"].cuda(), case["weight"].cuda()
    b, s, d = x.shape
    y = kf.rms_norm(b, s, d, case["eps"], str(x.dtype).removeprefix("torch."))(x, w)
    assert y.shape == case["y"].shape and y.dtype == case["y"].dtype
    _check(y, case["y"])
    if y.dtype != torch.float32:
        assert_rmsnorm_stated_bar(y.cpu(), oracle.rmsnorm_forward(case["x"], None, case["eps"]), case["weight"])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("shape", [(8, 512, 1024), (1, 4096, 2048), (2, 33, 4096), (1, 7, 8192),
                                   (3, 5, 1000), (1, 3, 77), (2, 2, 16384), (1, 2, 40000), (1, 9, 8)])
def test_against_oracle(kf, shape, dtype):
    g = torch.Generator().manual_seed(sum(shape) * 7 + {torch.bfloat16: 1, torch.float16: 2, torch.float32: 3}[dtype])
    x = torch.randn(shape, generator=g).to(dtype)
    w = (1 + 0.1 * torch.randn(shape[-1], generator=g)).to(dtype)
    from kernelforge_b200.rmsnorm.custom import rmsnorm_forward

    y = rmsnorm_forward(x.cuda(), w.cuda(), 1e-6)
    _check(y, oracle.rmsnorm_forward(x, w, 1e-6))
    if dtype != torch.float32:
        # The weightless normalised row has a single rounding: within 1 ulp.
        assert_within_ulps(rmsnorm_forward(x.cuda(), None, 1e-6), oracle.rmsnorm_forward(x, None, 1e-6), ulps=1)
        # The stated bar (1 ulp + 1e-2), double-rounding neighbours aside.
        assert_rmsnorm_stated_bar(y.cpu(), oracle.rmsnorm_forward(x, None, 1e-6), w)


def test_reference_harness_form(kf):
    """rmsnorm/test.py:38-63: seed 0, bf16, weight = randn, rtol = atol = 2e-2 (and 1 ulp here)."""
    torch.manual_seed(0)
    x = torch.randn(8, 512, 1024, device="cuda", dtype=torch.bfloat16)
    weight = torch.randn(1024, device="cuda", dtype=torch.bfloat16)
    out = kf.custom_rms_norm(batch=8, seq_len=512, dim=1024, eps=1e-6, dtype="bfloat16")(x, weight)
    expected = oracle.rmsnorm_forward(x.cpu(), weight.cpu(), 1e-6)
    torch.testing.assert_close(out.float().cpu(), expected.float(), rtol=2e-2, atol=2e-2)
    assert_rmsnorm_close(out, expected)


def test_strided_misaligned_and_weightless(kf):
    from kernelforge_b200.rmsnorm.custom import rmsnorm_forward

    g = torch.Generator().manual_seed(7)
    wide = torch.randn(64, 2056, generator=g).to(torch.bfloat16).cuda()
    x = wide[:, :2048]                       # row stride 2056 (vector path, strided rows)
    w = (1 + 0.1 * torch.randn(2048, generator=g)).to(torch.bfloat16).cuda()
    _check(rmsnorm_forward(x, w, 1e-6), oracle.rmsnorm_forward(x.cpu(), w.cpu(), 1e-6))
    shifted = wide.reshape(-1)[1:1 + 64 * 2048].view(64, 2048)  # 2-byte aligned only -> generic path
    _check(rmsnorm_forward(shifted, w, 1e-6), oracle.rmsnorm_forward(shifted.cpu(), w.cpu(), 1e-6))
    a = torch.randn(37, 4096, generator=g).cuda()
    _check(kf.original_tilelang_rms_norm(a, 1), oracle.rmsnorm_forward(a.cpu(), None, 1e-12))


def test_empty_and_module(kf):
    from kernelforge_b200.rmsnorm.custom import rmsnorm_forward

    empty = torch.empty(0, 1024, dtype=torch.bfloat16, device="cuda")
    assert rmsnorm_forward(empty, torch.ones(1024, dtype=torch.bfloat16, device="cuda")).shape == (0, 1024)
    m = kf.RMSNorm(256).cuda()  # fp32 weight with bf16 input: torch type promotion, as the reference
    x = torch.randn(4, 256, device="cuda").to(torch.bfloat16)
    ref_mod_out = oracle.rmsnorm_forward(x.cpu(), None, 1e-6) * m.weight.detach().cpu()
    out = m(x)
    assert out.dtype == torch.float32
    torch.testing.assert_close(out.cpu(), ref_mod_out, rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("rows,hidden", [(4096, 1024), (32768, 4096), (262144, 8192)])
def test_baseline_sweep_points(kf, rows, hidden):
    """BASELINE sweep shapes: sampled rows against the CPU oracle, every row against a
    chunked fp32 torch evaluation on the GPU (1 ulp)."""
    from kernelforge_b200.rmsnorm.custom import rmsnorm_forward

    g = torch.Generator(device="cuda").manual_seed(rows + hidden)
    x = torch.randn(rows, hidden, device="cuda", generator=g, dtype=torch.float32).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(hidden, device="cuda", generator=g)).to(torch.bfloat16)
    y = rmsnorm_forward(x, w, 1e-6)
    sample = torch.randint(0, rows, (64,), generator=torch.Generator().manual_seed(1))
    assert_rmsnorm_close(y[sample.cuda()], oracle.rmsnorm_forward(x[sample.cuda()].cpu(), w.cpu(), 1e-6))
    chunk = 16384
    mismatched = 0
    for r0 in range(0, rows, chunk):
        xs = x[r0:r0 + chunk].float()
        r = 1.0 / torch.sqrt(xs.pow(2).mean(-1, keepdim=True) + 1e-6)
        normed = (xs * r).to(torch.bfloat16)
        ref = (normed.float() * w.float()).to(torch.bfloat16)
        dist = ulp_distance(y[r0:r0 + chunk], ref, torch.bfloat16)
        assert int(dist.max()) <= 2, f"rows {r0}..: max ulp distance {int(dist.max())}"
        mismatched += int((dist > 0).sum())
        # The stated bar, 1 ulp + 1e-2, on every element (double-rounding neighbours aside).
        assert_rmsnorm_stated_bar(y[r0:r0 + chunk], normed, w)
    # Differences come only from last-bit differences of the fp32 row scale: rare.
    assert mismatched < 1e-3 * rows * hidden, mismatched
    del x, y
    torch.cuda.empty_cache()


# ---------------------------------------------------------------------------------------------
# Backward (kf_rmsnorm_bwd). The reference's RMSNorm is forward-only; the oracle differentiates
# its forward in float64 (oracle.rmsnorm.rmsnorm_backward). dx is computed in fp32 and rounded
# once: within 1 ulp of the float64 value for 16-bit types (rtol 2^-8, doubled for the rounding
# of the fp32 value) or rtol 1e-4 for fp32, with atol 1e-3 (16-bit) / 1e-5 (fp32) of the largest
# |dx| for the cancellation in r g - x c. dweight sums rows in fp32: atol scaled by the sum of the
# terms' magnitudes.
# ---------------------------------------------------------------------------------------------
BWD_TOL = {torch.bfloat16: (8e-3, 1e-3), torch.float16: (1e-3, 1e-3), torch.float32: (1e-4, 1e-5)}


def _bwd_inputs(shape, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(shape, generator=g).to(dtype)
    w = (1 + 0.1 * torch.randn(shape[-1], generator=g)).to(dtype)
    dy = torch.randn(shape, generator=g).to(dtype)
    return x, w, dy


def _check_bwd(dx, dw, x, w, dy, eps):
    rtol, atol = BWD_TOL[x.dtype]
    ref_dx, ref_dw = oracle.rmsnorm_backward(x.cpu(), None if w is None else w.cpu(), dy.cpu(), eps)
    assert dx.dtype == x.dtype and dx.shape == x.shape
    torch.testing.assert_close(dx.cpu().double(), ref_dx, rtol=rtol, atol=atol * ref_dx.abs().max().item())
    if w is None:
        assert dw is None
        return
    xd = x.cpu().double()
    r = 1.0 / torch.sqrt((xd * xd).mean(-1, keepdim=True) + eps)
    mag = (dy.cpu().double().abs() * (xd * r).abs()).reshape(-1, x.shape[-1]).sum(0).max().item()
    assert dw.dtype == x.dtype and dw.shape == w.shape
    torch.testing.assert_close(dw.cpu().double(), ref_dw, rtol=rtol, atol=max(atol, 1e-5) * mag)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("shape", [(4, 256, 1024), (1, 3000, 4096), (2, 33, 8192), (1, 7, 2048), (3, 5, 1000),
                                   (1, 3, 77), (2, 2, 16384), (1, 9, 8), (1, 1, 4096), (640, 256)])
def test_backward_against_oracle(kf, shape, dtype):
    x, w, dy = _bwd_inputs(shape, dtype, sum(shape) + 11)
    dx, dw = kf.rmsnorm_backward(dy.cuda(), x.cuda(), w.cuda(), 1e-6)
    _check_bwd(dx, dw, x, w, dy, 1e-6)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_backward_weightless_strided_and_deterministic(kf, dtype):
    x, w, dy = _bwd_inputs((300, 2048), dtype, 5)
    dx, dw = kf.rmsnorm_backward(dy.cuda(), x.cuda(), None, 1e-5)
    _check_bwd(dx, dw, x, None, dy, 1e-5)
    # rows with a stride (a view of every other row of a wider buffer) and misaligned rows
    wide = torch.zeros(300, 2 * 2048 + 3, dtype=dtype, device="cuda")
    xv = wide[:, 3:2051]
    xv.copy_(x.cuda())
    dx2, dw2 = kf.rmsnorm_backward(dy.cuda(), xv, w.cuda(), 1e-5)
    _check_bwd(dx2, dw2, x, w, dy, 1e-5)
    dx3, dw3 = kf.rmsnorm_backward(dy.cuda(), x.cuda(), w.cuda(), 1e-5)
    dx4, dw4 = kf.rmsnorm_backward(dy.cuda(), x.cuda(), w.cuda(), 1e-5)
    assert torch.equal(dx3, dx4) and torch.equal(dw3, dw4)  # fixed summation order


def test_backward_empty_and_autograd(kf):
    w = torch.ones(512, dtype=torch.bfloat16, device="cuda")
    empty = torch.empty(0, 512, dtype=torch.bfloat16, device="cuda")
    dx, dw = kf.rmsnorm_backward(empty, empty, w, 1e-6)
    assert dx.shape == (0, 512) and torch.count_nonzero(dw) == 0
    # autograd through the module and the Function: same gradients as the oracle
    x, w16, dy = _bwd_inputs((2, 64, 1024), torch.bfloat16, 21)
    m = kf.RMSNorm(1024).cuda().to(torch.bfloat16)
    with torch.no_grad():
        m.weight.copy_(w16.cuda())
    xg = x.cuda().requires_grad_()
    m(xg).backward(dy.cuda())
    _check_bwd(xg.grad, m.weight.grad, x, w16, dy, 1e-6)
    # fp32 weight with bf16 input: the kernel's weightless normalisation, then torch's promotion
    m32 = kf.RMSNorm(1024).cuda()
    xg = x.cuda().requires_grad_()
    out = m32(xg)
    out.backward(torch.ones_like(out))
    ref_dx, _ = oracle.rmsnorm_backward(x, None, torch.ones_like(x), 1e-6)
    torch.testing.assert_close(xg.grad.cpu().double(), ref_dx, rtol=8e-3, atol=1e-3 * ref_dx.abs().max().item())
    assert m32.weight.grad is not None and m32.weight.grad.dtype == torch.float32


def test_backward_large_rows_vs_fp32_torch(kf):
    """The BASELINE sweep's largest hidden size over many rows: every row against an fp32 torch
    evaluation on the GPU."""
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn(32768, 8192, device="cuda", generator=g).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(8192, device="cuda", generator=g)).to(torch.bfloat16)
    dy = torch.randn(32768, 8192, device="cuda", generator=g).to(torch.bfloat16)
    dx, dw = kf.rmsnorm_backward(dy, x, w, 1e-6)
    xf, wf, dyf = x.float(), w.float(), dy.float()
    r = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6)
    gf = dyf * wf
    ref_dx = r * gf - xf * r.pow(3) * (gf * xf).sum(-1, keepdim=True) / 8192
    ref_dw = (dyf * (xf * r).to(torch.bfloat16).float()).sum(0)
    torch.testing.assert_close(dx.float(), ref_dx, rtol=8e-3, atol=1e-3 * ref_dx.abs().max().item())
    mag = (dyf.abs() * (xf * r).abs()).sum(0).max().item()
    torch.testing.assert_close(dw.float(), ref_dw, rtol=8e-3, atol=1e-5 * mag)
