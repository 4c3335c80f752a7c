"""kf_sana_linattn_fwd_noalloc: the SANA attention entry point for callers that cannot allocate
device memory (its scratch is a fixed device array inside the library).

Called through the C ABI and checked against the workspace entry point kf_sana_linattn_fwd on
the same inputs, with the SANA tolerance (bf16 out: 1 ulp + atol 2e-3; fp32 out: rtol 1e-4),
on two calls in a row, on both the head_dim-32 fast path and the generic path (whose arrival
counters the no-alloc call must zero itself). Collected last so that a run stopping at its
first failure has already run every other test; it also passes alone in a fresh process.
"""

import pytest
import torch

from tests.tolerances import assert_close_ulp_atol

pytestmark = pytest.mark.gpu

CODES = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("CUDA is required")
    from kernelforge_b200 import _lib

    return _lib


def _workspace_call(lib, qkv, out, heads, dim):
    b, n = qkv.shape[0], qkv.shape[1]
    size = lib.lib.kf_sana_linattn_workspace_size(b, heads, dim, n, 0)
    ws = torch.zeros(size, dtype=torch.uint8, device=qkv.device)
    rc = lib.lib.kf_sana_linattn_fwd(qkv.data_ptr(), out.data_ptr(), ws.data_ptr(), size, b, heads, dim, n, 0,
                                     1e-15, CODES[qkv.dtype], CODES[out.dtype],
                                     lib.stream_handle(qkv.device))
    assert rc == 0, lib.status_string(rc)
    return out


def _noalloc_call(lib, qkv, out, heads, dim):
    b, n = qkv.shape[0], qkv.shape[1]
    rc = lib.lib.kf_sana_linattn_fwd_noalloc(qkv.data_ptr(), out.data_ptr(), b, heads, dim, n, 0, 1e-15,
                                             CODES[qkv.dtype], CODES[out.dtype], lib.stream_handle(qkv.device))
    assert rc == 0, lib.status_string(rc)
    return out


def _compare(actual, expected):
    if expected.dtype == torch.float32:
        torch.testing.assert_close(actual.cpu(), expected.cpu(), rtol=1e-4, atol=1e-5)
    else:
        assert_close_ulp_atol(actual, expected, dtype=expected.dtype, ulps=1, atol=2e-3)


@pytest.mark.parametrize(
    "b,n,heads,dim,in_dtype,out_dtype",
    [
        (2, 1000, 6, 32, torch.bfloat16, torch.bfloat16),  # fast path (TMA + cluster reduction)
        (1, 4096, 36, 32, torch.float16, torch.float32),   # fast path, fp16 operand scaling
        (2, 300, 4, 64, torch.float32, torch.float32),     # generic path (partials + counters)
    ],
)
def test_noalloc_matches_workspace_entry_point(lib, b, n, heads, dim, in_dtype, out_dtype):
    g = torch.Generator().manual_seed(b * 7919 + n + heads + dim)
    device = torch.device("cuda", 0)
    for call in range(2):  # two calls in a row: the shared scratch keeps the previous contents
        qkv = torch.randn(b, n, 3, heads * dim, generator=g).to(in_dtype).to(device)
        expected = _workspace_call(lib, qkv, torch.empty(b, n, heads * dim, dtype=out_dtype, device=device), heads, dim)
        actual = _noalloc_call(lib, qkv, torch.empty(b, n, heads * dim, dtype=out_dtype, device=device), heads, dim)
        torch.cuda.synchronize()
        _compare(actual, expected)
        assert torch.isfinite(actual).all(), f"call {call}"
    assert lib.query_device_error(device) == 0


def test_noalloc_rejects_shapes_beyond_the_scratch(lib):
    limit = lib.lib.kf_sana_noalloc_scratch_bytes()
    assert limit == 16 << 20
    heads = 64
    batch = limit // (heads * 33 * 32 * 4) + 1  # one more (batch, head) block than fits
    tiny = torch.zeros(16, dtype=torch.bfloat16, device="cuda")
    rc = lib.lib.kf_sana_linattn_fwd_noalloc(tiny.data_ptr(), tiny.data_ptr(), batch, heads, 32, 4096, 0, 1e-15,
                                             2, 2, lib.stream_handle(tiny.device))
    assert rc == 4, lib.status_string(rc)  # KF_ERR_WORKSPACE, before any launch
