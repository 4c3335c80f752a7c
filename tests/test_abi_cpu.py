"""C ABI checks that need no GPU: the library loads and exports every declared symbol, and the
host-side argument validation rejects bad calls before any launch."""

import ctypes
import re
from pathlib import Path

import pytest
import torch

from kernelforge_b200 import _lib

HEADER = Path(__file__).resolve().parent.parent / "include" / "kernelforge_b200.h"


def declared_functions():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(kf_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared_functions()
    assert "kf_rmsnorm_fwd" in names and "kf_sana_linattn_fwd" in names


@pytest.mark.parametrize("name", declared_functions())
def test_library_exports_declared_symbol(name):
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    assert hasattr(lib, name), f"{name} is declared in {HEADER.name} but not exported"
    assert name in _lib.SIGNATURES, f"{name} has no ctypes signature in kernelforge_b200/_lib.py"


def test_status_strings_and_version():
    assert _lib.status_string(0) == "ok"
    assert "workspace" in _lib.status_string(4)
    assert _lib.lib.kf_abi_version() >= 2


def test_rmsnorm_rejects_bad_arguments_without_launching():
    f = _lib.lib.kf_rmsnorm_fwd
    # bad dtype / sizes / null pointers are refused before touching the device
    assert f(1, None, 1, 4, 8, 8, 8, 1e-6, 7, None) == 2
    assert f(1, None, 1, 4, 0, 8, 8, 1e-6, 2, None) == 1
    assert f(None, None, 1, 4, 8, 8, 8, 1e-6, 2, None) == 1
    assert f(16, None, 16, 4, 8, 4, 8, 1e-6, 2, None) == 1  # row stride < dim
    assert f(17, None, 16, 4, 8, 8, 8, 1e-6, 2, None) == 3  # misaligned bf16 pointer
    assert f(None, None, None, 0, 8, 8, 8, 1e-6, 2, None) == 0  # empty: no-op


def test_sana_workspace_and_validation():
    ws = _lib.lib.kf_sana_linattn_workspace_size
    assert ws(4, 36, 32, 4096, 0) > 0
    assert ws(4, 36, 48, 4096, 0) == 0  # 48 does not divide 128
    # more splits never shrink the workspace
    assert ws(2, 70, 32, 16384, 16) >= ws(2, 70, 32, 16384, 1)
    f = _lib.lib.kf_sana_linattn_fwd
    need = ws(1, 2, 32, 128, 0)
    assert f(256, 256, 256, need - 1, 1, 2, 32, 128, 0, 1e-15, 2, 2, None) == 4  # workspace too small
    assert f(256, 256, 256, need, 1, 2, 24, 128, 0, 1e-15, 2, 2, None) == 2      # head dim
    assert f(256, 256, None, need, 1, 2, 32, 128, 0, 1e-15, 2, 2, None) == 1     # no workspace
    assert f(256, 256, 256, need, 1, 2, 32, 128, 0, 1e-15, 5, 2, None) == 2      # dtype


def test_linear_validation_without_launching():
    f = _lib.lib.kf_linear_fwd
    # x, weight, bias, y, rows, in, out, layout, dtype, stream
    assert f(256, 256, None, 256, 4, 8, 8, 0, 7, None) == 2      # dtype
    assert f(None, 256, None, 256, 4, 8, 8, 0, 2, None) == 1     # no x
    assert f(256, 256, None, 256, 4, 8, 8, 2, 2, None) == 1      # weight layout
    assert f(256, 256, None, 256, 4, 0, 8, 0, 2, None) == 1      # in_features
    assert f(256, 256, None, 256, 4, 8, 12, 0, 2, None) == 2     # 16-bit out_features % 8
    assert f(256, 256, None, 264 + 2, 4, 8, 8, 1, 1, None) == 3  # misaligned y
    assert f(256, 256, 258, 256, 4, 8, 8, 0, 2, None) == 3       # misaligned bias
    assert f(256, 256, None, 256, 0, 8, 8, 0, 2, None) == 0      # no rows: no-op
    assert f(None, None, None, None, 0, 8, 8, 0, 2, None) == 0   # ... whatever the pointers


def test_fa_bwd_workspace_and_validation():
    ws = _lib.lib.kf_fa_bwd_workspace_size
    # Two fp32 statistics per (batch, head, query), padded to 128 queries; the fused schedule
    # (deterministic=0, head dim <= 128) adds the fp32 dQ sums, 64 or 128 per row.
    assert ws(2, 4, 100, 64, 1) == 2 * 2 * 4 * 128 * 4
    assert ws(2, 4, 100, 256, 0) == 2 * 2 * 4 * 128 * 4
    assert ws(2, 4, 100, 40, 0) == (2 + 64) * 2 * 4 * 128 * 4
    assert ws(2, 4, 100, 96, 0) == (2 + 128) * 2 * 4 * 128 * 4
    assert ws(0, 4, 100, 64, 0) == 0
    assert ws(1, 4, 100, 0, 0) == 0
    f = _lib.lib.kf_fa_bwd
    need = ws(1, 2, 16, 64, 0)
    ptrs = [256] * 9  # q, k, v, out, dout, lse, dq, dk, dv
    args = (1, 16, 16, 2, 2, 64, 0.125, 0, 0, 2, None)
    assert f(*ptrs, 256, need - 1, *args) == 4                                       # workspace too small
    assert f(*ptrs, 256, ws(1, 2, 16, 64, 1), *args) == 4                           # sized for deterministic
    assert f(*ptrs, None, need, *args) == 1                                          # no workspace
    assert f(*ptrs[:6], None, *ptrs[7:], 256, need, *args) == 1                      # no dq
    assert f(*ptrs[:4], 264, *ptrs[5:], 256, need, *args) == 3                       # misaligned dout
    assert f(*ptrs, 256, need, 1, 16, 16, 2, 2, 72 * 4, 0.125, 0, 0, 2, None) == 2   # head dim > 256
    assert f(*ptrs, 256, need, 1, 16, 16, 3, 2, 64, 0.125, 0, 0, 2, None) == 2      # Hq % Hkv
    assert f(*ptrs, 256, need, 1, 16, 16, 2, 2, 64, -1.0, 0, 0, 2, None) == 1       # scale
    assert f(*ptrs, 256, need, 1, 16, 16, 2, 2, 64, 0.125, 0, 0, 7, None) == 2      # dtype


def test_python_signature_validation():
    from kernelforge_b200.SANA_LinearAttention import qkv_attn_matmul
    from kernelforge_b200.rmsnorm import rms_norm

    with pytest.raises(ValueError, match="dim must divide"):
        qkv_attn_matmul(1, 2, 48, 128)
    with pytest.raises(ValueError, match="output_dtype"):
        qkv_attn_matmul(1, 2, 32, 128, output_dtype="int8")
    with pytest.raises(ValueError):
        rms_norm(0, 1, 8)
    kernel = rms_norm(1, 2, 8, 1e-6, "bfloat16")
    with pytest.raises(ValueError, match="shape"):
        kernel(torch.zeros(1, 3, 8, dtype=torch.bfloat16), torch.zeros(8, dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="CUDA"):
        kernel(torch.zeros(1, 2, 8, dtype=torch.bfloat16), torch.zeros(8, dtype=torch.bfloat16))


def test_rmsnorm_backward_validation_without_launching():
    ws = _lib.lib.kf_rmsnorm_bwd_workspace_size
    assert ws(8192) == 320 * 8192 * 4 and ws(0) == 0
    f = _lib.lib.kf_rmsnorm_bwd
    need = ws(64)
    # x, weight, dy, dx, dweight, workspace, workspace_bytes, rows, dim, strides, eps, dtype, stream
    assert f(256, 256, 256, 256, 256, 256, need, 4, 64, 64, 64, 64, 1e-6, 7, None) == 2      # dtype
    assert f(256, 256, 256, 256, 256, 256, need, -1, 64, 64, 64, 64, 1e-6, 2, None) == 1     # rows
    assert f(256, 256, 256, 256, None, 256, need, 4, 64, 64, 64, 64, 1e-6, 2, None) == 1    # weight without dweight
    assert f(256, 256, 256, 256, 256, 256, need - 1, 4, 64, 64, 64, 64, 1e-6, 2, None) == 4  # workspace
    assert f(256, 256, 256, 256, 256, None, need, 4, 64, 64, 64, 64, 1e-6, 2, None) == 1    # no workspace
    assert f(256, 256, 256, 256, 256, 256, need, 4, 64, 32, 64, 64, 1e-6, 2, None) == 1     # stride < dim
    assert f(257, 256, 256, 256, 256, 256, need, 4, 64, 64, 64, 64, 1e-6, 2, None) == 3     # misaligned bf16


def test_sana_plan_validation_without_launching():
    f = _lib.lib.kf_sana_linattn_plan
    launches, ctas = ctypes.c_int64(-1), ctypes.c_int64(-1)
    assert f(1, 36, 32, 4096, 0, 2, None, ctypes.byref(ctas)) == 1                          # no output
    assert f(1, 36, 32, 4096, 0, 7, ctypes.byref(launches), ctypes.byref(ctas)) == 2         # dtype
    assert f(0, 36, 32, 4096, 0, 2, ctypes.byref(launches), ctypes.byref(ctas)) == 1         # batch
    assert f(1, 36, 48, 4096, 0, 2, ctypes.byref(launches), ctypes.byref(ctas)) == 2         # head dim
    assert launches.value == -1 and ctas.value == -1                                          # nothing written
