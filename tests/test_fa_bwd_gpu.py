"""FlashAttention backward (reverse-mode VJP) parity on the GPU through the C ABI.

FlashAttentionFunction.backward hands dout and the saved (q, k, v, out, lse) to
``_flash_attn_backward`` (flash_attention_jvp/custom.py:255-266), which this library serves with
its own tcgen05 kernels: by default (``deterministic=False``, as the reference passes) one kernel
for head dims up to 128 whose dQ partials are summed at L2, else separate dQ and dK / dV
kernels with no atomics. Oracle: float64
autograd through the CPU attention restatement (``oracle.fa_jvp.attention``). Tolerances: the
reference harness's gradient bar (flash_attention_jvp/test.py:58-59; fp16 atol 3e-3 / rtol 1e-2,
bf16 atol = rtol = 3e-2) with atol scaled by the largest reference gradient, since dK / dV sum
over every query of a KV group.
"""

import pytest
import torch

from oracle.fa_jvp import attention
from tests.tolerances import fa_tolerance

pytestmark = pytest.mark.gpu
DTYPES = (torch.float16, torch.bfloat16)
# B, Nq, Nk, Hq, Hkv, D, causal, scale
CASES = (
    (1, 7, 11, 2, 2, 8, False, None),
    (2, 33, 65, 4, 4, 24, False, 0.3),
    (1, 129, 131, 3, 3, 64, False, None),
    (1, 65, 65, 2, 2, 64, True, None),
    (1, 19, 71, 4, 2, 96, True, None),
    (1, 71, 19, 4, 1, 32, True, None),
    (1, 37, 91, 6, 2, 128, False, 0.2),
    (1, 9, 13, 2, 1, 256, False, None),
    (1, 1, 1, 2, 2, 64, True, None),
    (1, 17, 29, 2, 2, 16, False, 0.05),
    (1, 23, 37, 2, 2, 80, False, 0.15),
    (1, 300, 200, 4, 4, 192, True, None),
    (2, 256, 384, 8, 2, 128, True, None),
    (1, 200, 333, 2, 2, 256, True, 0.1),
    (1, 999, 515, 2, 2, 64, False, None),
    (2, 300, 200, 4, 2, 64, True, None),
    (1, 200, 450, 4, 1, 128, True, None),
    (1, 1000, 1000, 2, 2, 128, False, None),
    (3, 130, 70, 6, 3, 64, True, 0.3),
    (1, 300, 257, 4, 2, 96, True, None),
    (2, 129, 200, 2, 2, 72, False, 0.11),
    (1, 256, 256, 2, 1, 120, False, None),
)


@pytest.fixture(scope="module")
def fa():
    if not torch.cuda.is_available():
        pytest.skip("CUDA is required")
    import kernelforge_b200.flash_attention_jvp.custom as mod

    return mod


def make_inputs(case, dtype, seed=2027):
    b, nq, nk, h, hk, d, _, _ = case
    gen = torch.Generator(device="cpu").manual_seed(seed)
    shapes = ((b, nq, h, d), (b, nk, hk, d), (b, nk, hk, d), (b, nq, h, d))
    return tuple(torch.randn(s, generator=gen).to("cuda", dtype) for s in shapes)


def reference_grads(q, k, v, dout, causal, scale):
    primals = tuple(x.detach().cpu().double().requires_grad_() for x in (q, k, v))
    out = attention(*primals, causal=causal, softmax_scale=scale)
    return torch.autograd.grad(out, primals, dout.cpu().double())


def assert_grad_close(actual, expected, dtype):
    tol = fa_tolerance(dtype)
    scale = max(1.0, expected.abs().max().item())
    torch.testing.assert_close(actual.cpu().double(), expected, atol=tol["atol"] * scale, rtol=tol["rtol"])


def autograd_grads(fa, q, k, v, dout, causal, scale):
    primals = tuple(x.detach().requires_grad_() for x in (q, k, v))
    out = fa.flash_attention(*primals, causal=causal, softmax_scale=scale)
    return torch.autograd.grad(out, primals, dout)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("case", CASES)
def test_backward_matches_oracle(fa, case, dtype):
    q, k, v, dout = make_inputs(case, dtype)
    causal, scale = case[-2], case[-1]
    grads = autograd_grads(fa, q, k, v, dout, causal, scale)
    expected = reference_grads(q, k, v, dout, causal, scale)
    for name, actual, ref in zip(("dq", "dk", "dv"), grads, expected):
        assert actual.dtype == dtype and actual.shape == ref.shape, name
        assert torch.isfinite(actual).all(), name
        assert_grad_close(actual, ref, dtype)


def direct_grads(fa, q, k, v, dout, causal, scale, deterministic):
    out, lse = fa.flash_attention(q, k, v, causal=causal, softmax_scale=scale, return_lse=True)
    grads = tuple(torch.full_like(x, float("nan")) for x in (q, k, v))
    used = q.shape[-1] ** -0.5 if scale is None else scale
    fa._flash_attn_backward(dout, q, k, v, out, lse, *grads, 0.0, used, causal, deterministic=deterministic)
    return grads


def assert_dq_close(actual, expected):
    """The fused schedule's dq against the deterministic one: the same fp32 terms summed in
    another order, then rounded to 16 bits, so at most a unit or so in the last place apart."""
    scale = expected.abs().max().item()
    torch.testing.assert_close(actual.float(), expected.float(), rtol=2 ** -7, atol=1e-4 * scale)


@pytest.mark.parametrize("dtype", DTYPES)
def test_backward_is_deterministic(fa, dtype):
    case = (2, 256, 320, 8, 2, 64, True, None)
    q, k, v, dout = make_inputs(case, dtype)
    first = direct_grads(fa, q, k, v, dout, True, None, deterministic=True)
    second = direct_grads(fa, q, k, v, dout, True, None, deterministic=True)
    for a, b in zip(first, second):
        assert torch.equal(a, b)
    # The default (fused) schedule: dK and dV are summed in a fixed order, dQ at L2.
    fast = direct_grads(fa, q, k, v, dout, True, None, deterministic=False)
    again = direct_grads(fa, q, k, v, dout, True, None, deterministic=False)
    for a, b in zip(fast[1:], again[1:]):
        assert torch.equal(a, b)
    assert_dq_close(again[0], fast[0])


FUSED_CASES = tuple(c for c in CASES if c[5] <= 128) + (
    (2, 1000, 777, 8, 2, 128, True, None),
    (1, 513, 1031, 4, 4, 64, False, None),
    (4, 128, 128, 16, 16, 128, False, None),
)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("case", FUSED_CASES)
def test_fused_schedule_matches_deterministic(fa, case, dtype):
    """Head dims up to 128: the one-kernel schedule's dK and dV equal the separate kernels' bit
    for bit (same tiles, same MMA order); dQ agrees to the last place."""
    q, k, v, dout = make_inputs(case, dtype, seed=77)
    causal, scale = case[-2], case[-1]
    fast = direct_grads(fa, q, k, v, dout, causal, scale, deterministic=False)
    exact = direct_grads(fa, q, k, v, dout, causal, scale, deterministic=True)
    assert torch.equal(fast[1], exact[1]) and torch.equal(fast[2], exact[2])
    assert torch.isfinite(fast[0]).all()
    assert_dq_close(fast[0], exact[0])


def test_direct_call_writes_in_place_and_strided_destinations(fa):
    case = (1, 67, 41, 4, 2, 64, True, 0.17)
    q, k, v, dout = make_inputs(case, torch.bfloat16)
    out, lse = fa.flash_attention(q, k, v, causal=True, softmax_scale=0.17, return_lse=True)
    dq, dk, dv = (torch.full_like(x, float("nan")) for x in (q, k, v))
    ret = fa._flash_attn_backward(dout, q, k, v, out, lse, dq, dk, dv, 0.0, 0.17, True)
    assert ret[0] is dq and ret[1] is dk and ret[2] is dv
    expected = reference_grads(q, k, v, dout, True, 0.17)
    for actual, ref in zip((dq, dk, dv), expected):
        assert_grad_close(actual, ref, torch.bfloat16)
    # Strided destinations (a view into a wider buffer) receive the same values.
    wide = tuple(torch.zeros((*x.shape[:-1], 2 * x.shape[-1]), device="cuda", dtype=x.dtype) for x in (q, k, v))
    views = tuple(w[..., ::2] for w in wide)
    fa._flash_attn_backward(dout, q, k, v, out, lse, *views, 0.0, 0.17, True)
    for view, dense in zip(views, (dq, dk, dv)):
        assert torch.equal(view, dense)
    with pytest.raises(NotImplementedError):
        fa._flash_attn_backward(dout, q, k, v, out, lse, dq, dk, dv, 0.1, 0.17, True)


def test_fully_masked_rows_and_keys_get_zero_gradients(fa):
    # Causal with Nq > Nk: the first Nq - Nk queries see no key (bottom-right alignment).
    case = (1, 90, 40, 2, 1, 64, True, None)
    q, k, v, dout = make_inputs(case, torch.float16)
    dq, dk, dv = autograd_grads(fa, q, k, v, dout, True, None)
    assert torch.count_nonzero(dq[:, : 90 - 40]) == 0
    expected = reference_grads(q, k, v, dout, True, None)
    for actual, ref in zip((dq, dk, dv), expected):
        assert_grad_close(actual, ref, torch.float16)


def test_gqa_group_sum_equals_repeated_heads(fa):
    # dK / dV of a shared KV head are the sum over its query heads: compare with MHA on
    # repeated K / V and a group sum of the per-head gradients.
    case = (1, 130, 150, 8, 2, 128, False, None)
    q, k, v, dout = make_inputs(case, torch.bfloat16)
    dq, dk, dv = autograd_grads(fa, q, k, v, dout, False, None)
    rk, rv = (x.repeat_interleave(4, dim=2) for x in (k, v))
    dq_r, dk_r, dv_r = autograd_grads(fa, q, rk, rv, dout, False, None)
    assert_dq_close(dq, dq_r)
    exact = direct_grads(fa, q, k, v, dout, False, None, deterministic=True)
    exact_r = direct_grads(fa, q, rk, rv, dout, False, None, deterministic=True)
    torch.testing.assert_close(exact[0], exact_r[0], atol=0, rtol=0)
    for grouped, repeated in ((dk, dk_r), (dv, dv_r)):
        summed = repeated.float().view(1, 150, 2, 4, 128).sum(3)
        torch.testing.assert_close(grouped.float(), summed, atol=3e-2, rtol=3e-2)


@pytest.mark.parametrize("deterministic", (True, False))
def test_backward_under_cuda_graph(fa, deterministic):
    case = (1, 128, 256, 4, 4, 64, False, None)
    q, k, v, dout = make_inputs(case, torch.float16)
    out, lse = fa.flash_attention(q, k, v, return_lse=True)
    dq, dk, dv = (torch.empty_like(x) for x in (q, k, v))
    args = (dout, q, k, v, out, lse, dq, dk, dv, 0.0, 0.125, False)
    fa._flash_attn_backward(*args, deterministic=deterministic)
    torch.cuda.synchronize()
    eager = tuple(x.clone() for x in (dq, dk, dv))
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        fa._flash_attn_backward(*args, deterministic=deterministic)
        with torch.cuda.graph(graph, stream=stream):
            fa._flash_attn_backward(*args, deterministic=deterministic)
    torch.cuda.current_stream().wait_stream(stream)
    for x in (dq, dk, dv):
        x.zero_()
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(dk, eager[1]) and torch.equal(dv, eager[2])
    if deterministic:
        assert torch.equal(dq, eager[0])
    else:
        assert_dq_close(dq, eager[0])
    del graph
