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
from tests.tolerances import assert_rmsnorm_close, assert_within_ulps, ulp_distance

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
        ref = ((xs * r).to(torch.bfloat16).float() * w.float()).to(torch.bfloat16)
        dist = ulp_distance(y[r0:r0 + chunk], ref, torch.bfloat16)
        assert int(dist.max()) <= 2, f"rows {r0}..: max ulp distance {int(dist.max())}"
        mismatched += int((dist > 0).sum())
    # Differences come only from last-bit differences of the fp32 row scale: rare.
    assert mismatched < 1e-3 * rows * hidden, mismatched
    del x, y
    torch.cuda.empty_cache()
