"""kf_sana_linattn_fwd_noalloc: the SANA attention entry point for callers that cannot allocate
device memory (its scratch is a fixed device array inside the library).

Called through the C ABI and checked against the workspace entry point kf_sana_linattn_fwd on
the same inputs, with the SANA tolerance (bf16 out: 1 ulp + atol 2e-3; fp32 out: rtol 1e-4),
on two calls in a row, on the head_dim-32 split path, the one-launch path (which needs no
scratch), the generic path (whose arrival counters the no-alloc call must zero itself), and on
split counts lowered to fit the array. One case runs in a child process without torch: a call,
then cudaDeviceReset, then a call in the new context, whose array address must be looked up
again. Collected last so that a run stopping at its first failure has already run every other
test; it also passes alone in a fresh process.
"""

import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

from tests.tolerances import assert_close_ulp_atol

pytestmark = pytest.mark.gpu

CODES = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}
ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("CUDA is required")
    from kernelforge_b200 import _lib

    return _lib


def _workspace_call(lib, qkv, out, heads, dim, splits=0):
    b, n = qkv.shape[0], qkv.shape[1]
    size = lib.lib.kf_sana_linattn_workspace_size(b, heads, dim, n, splits)
    ws = torch.zeros(size, dtype=torch.uint8, device=qkv.device)
    rc = lib.lib.kf_sana_linattn_fwd(qkv.data_ptr(), out.data_ptr(), ws.data_ptr(), size, b, heads, dim, n, splits,
                                     1e-15, CODES[qkv.dtype], CODES[out.dtype],
                                     lib.stream_handle(qkv.device))
    assert rc == 0, lib.status_string(rc)
    return out


def _noalloc_call(lib, qkv, out, heads, dim, splits=0):
    b, n = qkv.shape[0], qkv.shape[1]
    rc = lib.lib.kf_sana_linattn_fwd_noalloc(qkv.data_ptr(), out.data_ptr(), b, heads, dim, n, splits, 1e-15,
                                             CODES[qkv.dtype], CODES[out.dtype], lib.stream_handle(qkv.device))
    assert rc == 0, lib.status_string(rc)
    return out


def _compare(actual, expected):
    if expected.dtype == torch.float32:
        torch.testing.assert_close(actual.cpu(), expected.cpu(), rtol=1e-4, atol=1e-5)
    else:
        assert_close_ulp_atol(actual, expected, dtype=expected.dtype, ulps=1, atol=2e-3)


def _split_bytes(b, heads, dim, splits):
    """Scratch of the split paths for `splits` chunks (the layouts of sana_linattn.cu)."""
    counters = (b * heads * 4 + 255) // 256 * 256
    if dim == 32:
        return counters + (b * heads * splits * 33 * 32 * 4 + 255) // 256 * 256
    per_head = (dim + 1) * dim * 4
    return counters + (b * heads * splits * per_head + 255) // 256 * 256 + (b * heads * per_head + 255) // 256 * 256


@pytest.mark.parametrize(
    "b,n,heads,dim,in_dtype,out_dtype,splits",
    [
        (2, 1000, 6, 32, torch.bfloat16, torch.bfloat16, 0),   # automatic: split path, default splits
        (1, 4096, 36, 32, torch.float16, torch.float32, 0),    # split path, fp16 operand scaling
        (4, 1024, 36, 32, torch.bfloat16, torch.bfloat16, 0),  # automatic: one-launch path (no scratch)
        (2, 640, 6, 32, torch.bfloat16, torch.float32, -1),    # one-launch path forced (clusters)
        (2, 300, 4, 64, torch.float32, torch.float32, 0),      # generic path (partials + counters)
    ],
)
def test_noalloc_matches_workspace_entry_point(lib, b, n, heads, dim, in_dtype, out_dtype, splits):
    g = torch.Generator().manual_seed(b * 7919 + n + heads + dim)
    device = torch.device("cuda", 0)
    for call in range(2):  # two calls in a row: the shared scratch keeps the previous contents
        qkv = torch.randn(b, n, 3, heads * dim, generator=g).to(in_dtype).to(device)
        expected = _workspace_call(lib, qkv, torch.empty(b, n, heads * dim, dtype=out_dtype, device=device),
                                   heads, dim, splits)
        actual = _noalloc_call(lib, qkv, torch.empty(b, n, heads * dim, dtype=out_dtype, device=device),
                               heads, dim, splits)
        torch.cuda.synchronize()
        _compare(actual, expected)
        assert torch.isfinite(actual).all(), f"call {call}"
    assert lib.query_device_error(device) == 0


@pytest.mark.parametrize(
    "b,n,heads,dim,in_dtype,splits",
    [
        # Generic path, fp32, head_dim 128: the default split count (37 for 8 units on 148 SMs)
        # needs more than the 16 MiB array, so the call runs with fewer splits.
        (1, 4096, 8, 128, torch.float32, 0),
        # Fast split path with an explicit split count whose partials overflow the array.
        (8, 512, 64, 32, torch.bfloat16, 8),
    ],
)
def test_noalloc_lowers_split_count_to_fit(lib, b, n, heads, dim, in_dtype, splits):
    from oracle import sana as sana_oracle

    limit = lib.lib.kf_sana_noalloc_scratch_bytes()
    requested = splits if splits > 0 else 37
    assert _split_bytes(b, heads, dim, requested) > limit  # the case really reaches the lowering
    g = torch.Generator().manual_seed(4242 + dim)
    device = torch.device("cuda", 0)
    out_dtype = torch.float32
    for call in range(2):
        qkv_cpu = torch.randn(b, n, 3, heads * dim, generator=g).to(in_dtype)
        qkv = qkv_cpu.to(device)
        expected = _workspace_call(lib, qkv, torch.empty(b, n, heads * dim, dtype=out_dtype, device=device),
                                   heads, dim, splits)
        actual = _noalloc_call(lib, qkv, torch.empty(b, n, heads * dim, dtype=out_dtype, device=device),
                               heads, dim, splits)
        torch.cuda.synchronize()
        _compare(actual, expected)
        exact = sana_oracle.attn_exact(qkv_cpu, heads, dim).float()
        torch.testing.assert_close(actual.cpu(), exact, rtol=1e-4, atol=1e-5)
    assert lib.query_device_error(device) == 0


def test_noalloc_rejects_shapes_beyond_the_scratch(lib):
    limit = lib.lib.kf_sana_noalloc_scratch_bytes()
    assert limit == 16 << 20
    heads = 64
    batch = limit // (heads * 33 * 32 * 4) + 1  # one more (batch, head) block than fits
    tiny = torch.zeros(16, dtype=torch.bfloat16, device="cuda")
    # splits = 1 forces the split path: even one split's partials do not fit.
    rc = lib.lib.kf_sana_linattn_fwd_noalloc(tiny.data_ptr(), tiny.data_ptr(), batch, heads, 32, 4096, 1, 1e-15,
                                             2, 2, lib.stream_handle(tiny.device))
    assert rc == 4, lib.status_string(rc)  # KF_ERR_WORKSPACE, before any launch


_RESET_CHILD = r"""
import ctypes, sys
import numpy as np

kf = ctypes.CDLL(sys.argv[1])
rt = ctypes.CDLL("libcudart.so.12")  # the runtime the library already loaded (same soname)
drv = ctypes.CDLL("libcuda.so.1")
P, I64 = ctypes.c_void_p, ctypes.c_int64
kf.kf_sana_linattn_fwd_noalloc.argtypes = [P, P, I64, I64, I64, I64, I64, ctypes.c_float, ctypes.c_int,
                                           ctypes.c_int, P]
kf.kf_sana_linattn_fwd.argtypes = [P, P, P, ctypes.c_size_t, I64, I64, I64, I64, I64, ctypes.c_float,
                                   ctypes.c_int, ctypes.c_int, P]
kf.kf_sana_linattn_workspace_size.restype = ctypes.c_size_t
kf.kf_sana_linattn_workspace_size.argtypes = [I64] * 5
kf.kf_query_device_error.argtypes = [P, ctypes.POINTER(ctypes.c_int)]
B, N, H, D, SPLITS = 1, 4096, 36, 32, 4          # head_dim-32 split path: uses the scratch
rng = np.random.default_rng(7)

def bf16_bits(x):
    u = x.astype(np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)

def check(rc, what):
    if rc != 0:
        raise SystemExit(f"{what} returned {rc}")

def malloc(nbytes):
    p = ctypes.c_void_p()
    check(rt.cudaMalloc(ctypes.byref(p), ctypes.c_size_t(nbytes)), "cudaMalloc")
    return p

def ctx_id():
    i = ctypes.c_ulonglong(0)
    return i.value if drv.cuCtxGetId(None, ctypes.byref(i)) == 0 else 0

def run_pair(host_qkv):
    qkv = malloc(host_qkv.nbytes)
    check(rt.cudaMemcpy(qkv, ctypes.c_void_p(host_qkv.ctypes.data), ctypes.c_size_t(host_qkv.nbytes), 1),
          "cudaMemcpy H2D")
    out_bytes = B * N * H * D * 4
    out_a, out_b = malloc(out_bytes), malloc(out_bytes)
    ws_bytes = kf.kf_sana_linattn_workspace_size(B, H, D, N, SPLITS)
    ws = malloc(ws_bytes)
    check(rt.cudaMemset(ws, 0, ctypes.c_size_t(ws_bytes)), "cudaMemset")
    check(kf.kf_sana_linattn_fwd(qkv, out_a, ws, ws_bytes, B, H, D, N, SPLITS, 1e-15, 2, 0, None), "workspace call")
    check(kf.kf_sana_linattn_fwd_noalloc(qkv, out_b, B, H, D, N, SPLITS, 1e-15, 2, 0, None), "noalloc call")
    check(rt.cudaDeviceSynchronize(), "cudaDeviceSynchronize")
    code = ctypes.c_int(0)
    check(kf.kf_query_device_error(None, ctypes.byref(code)), "kf_query_device_error")
    check(code.value, "device error word")
    a = np.empty(B * N * H * D, np.float32)
    b = np.empty_like(a)
    check(rt.cudaMemcpy(ctypes.c_void_p(a.ctypes.data), out_a, ctypes.c_size_t(out_bytes), 2), "cudaMemcpy D2H")
    check(rt.cudaMemcpy(ctypes.c_void_p(b.ctypes.data), out_b, ctypes.c_size_t(out_bytes), 2), "cudaMemcpy D2H")
    for p in (qkv, out_a, out_b, ws):
        check(rt.cudaFree(p), "cudaFree")
    if not np.isfinite(b).all() or not np.allclose(b, a, rtol=1e-4, atol=1e-5):
        raise SystemExit(f"noalloc differs from the workspace entry point: max {np.abs(a - b).max()}")

check(rt.cudaSetDevice(0), "cudaSetDevice")
host = bf16_bits(rng.standard_normal(B * N * 3 * H * D))
run_pair(host)
first = ctx_id()
check(rt.cudaDeviceReset(), "cudaDeviceReset")
check(rt.cudaSetDevice(0), "cudaSetDevice")
probe = malloc(256)  # the runtime creates the new primary context here
check(rt.cudaFree(probe), "cudaFree")
second = ctx_id()
if first == 0 or second == 0 or first == second:
    # Never launch with a possibly stale address: report instead.
    raise SystemExit(f"context ids before/after reset: {first}/{second}")
run_pair(bf16_bits(rng.standard_normal(B * N * 3 * H * D)))
print("reset ok", first, second)
"""


def test_noalloc_after_device_reset(lib):
    """A call, cudaDeviceReset, then calls in the new context: the array's address is looked up
    again in the new context (a cached address from the old one would point at unmapped memory).
    Runs in a child process that never touches torch, so the reset cannot invalidate this
    process's tensors."""
    res = subprocess.run([sys.executable, "-c", _RESET_CHILD, str(lib.LIB_PATH)], capture_output=True, text=True,
                         timeout=300, cwd=ROOT, env=dict(os.environ))
    assert res.returncode == 0, res.stdout + res.stderr
    assert "reset ok" in res.stdout
