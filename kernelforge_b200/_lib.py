"""ctypes binding of the C ABI (``include/kernelforge_b200.h``).

The shared library is the product's only compute path: importing this module loads it and
raises ``ImportError`` if it is missing (build it with ``python -m kernelforge_b200.build``).
There is no fallback to PyTorch or to the CPU.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

import torch

LIB_PATH = Path(os.environ.get("KERNELFORGE_B200_LIB", Path(__file__).resolve().parent / "_lib" / "libkernelforge_b200.so"))

DTYPE_CODES = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}
DTYPE_NAMES = {"float": torch.float32, "float32": torch.float32, "float16": torch.float16,
               "bfloat16": torch.bfloat16}

KF_OK = 0
KF_ERR_DEVICE_TIMEOUT = 6

_c_i64 = ctypes.c_int64
_c_ptr = ctypes.c_void_p

# name -> (restype, argtypes): must mirror include/kernelforge_b200.h exactly.
SIGNATURES = {
    "kf_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "kf_abi_version": (ctypes.c_int, []),
    "kf_query_device_error": (ctypes.c_int, [_c_ptr, ctypes.POINTER(ctypes.c_int)]),
    "kf_selftest_bounded_wait": (ctypes.c_int, [_c_ptr]),
    "kf_rmsnorm_fwd": (ctypes.c_int, [_c_ptr, _c_ptr, _c_ptr, _c_i64, _c_i64, _c_i64, _c_i64,
                                      ctypes.c_float, ctypes.c_int, _c_ptr]),
    "kf_rmsnorm_bwd_workspace_size": (ctypes.c_size_t, [_c_i64]),
    "kf_rmsnorm_bwd": (ctypes.c_int, [_c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, ctypes.c_size_t, _c_i64,
                                      _c_i64, _c_i64, _c_i64, _c_i64, ctypes.c_float, ctypes.c_int, _c_ptr]),
    "kf_sana_linattn_workspace_size": (ctypes.c_size_t, [_c_i64, _c_i64, _c_i64, _c_i64, _c_i64]),
    "kf_sana_linattn_fwd": (ctypes.c_int, [_c_ptr, _c_ptr, _c_ptr, ctypes.c_size_t, _c_i64, _c_i64,
                                           _c_i64, _c_i64, _c_i64, ctypes.c_float, ctypes.c_int,
                                           ctypes.c_int, _c_ptr]),
    "kf_sana_linattn_qknorm_workspace_size": (ctypes.c_size_t, [_c_i64, _c_i64, _c_i64, _c_i64, _c_i64]),
    "kf_sana_linattn_qknorm_fwd": (ctypes.c_int, [_c_ptr, _c_ptr, _c_ptr, ctypes.c_size_t, _c_i64, _c_i64, _c_i64,
                                                  _c_i64, _c_i64, ctypes.c_float, _c_ptr, _c_ptr, ctypes.c_float,
                                                  ctypes.c_int, ctypes.c_int, _c_ptr]),
    "kf_sana_linattn_fwd_noalloc": (ctypes.c_int, [_c_ptr, _c_ptr, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64,
                                                   ctypes.c_float, ctypes.c_int, ctypes.c_int, _c_ptr]),
    "kf_sana_noalloc_scratch_bytes": (ctypes.c_size_t, []),
    "kf_sana_linattn_plan": (ctypes.c_int, [_c_i64, _c_i64, _c_i64, _c_i64, _c_i64, ctypes.c_int,
                                            ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(ctypes.c_int64)]),
    "kf_linear_fwd": (ctypes.c_int, [_c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_i64, _c_i64, _c_i64, ctypes.c_int,
                                     ctypes.c_int, _c_ptr]),
    "kf_sana_proj_attn_workspace_size": (ctypes.c_size_t, [_c_i64, _c_i64, _c_i64]),
    "kf_sana_proj_attn_fwd": (ctypes.c_int, [_c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, ctypes.c_size_t, _c_i64, _c_i64,
                                             _c_i64, ctypes.c_float, ctypes.c_int, _c_ptr]),
    "kf_fa_fwd": (ctypes.c_int, [_c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_i64, _c_i64, _c_i64, _c_i64,
                                 _c_i64, _c_i64, ctypes.c_float, ctypes.c_int, ctypes.c_int, _c_ptr]),
    "kf_fa_jvp": (ctypes.c_int, [_c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr,
                                 _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, ctypes.c_float,
                                 ctypes.c_int, ctypes.c_int, _c_ptr]),
    "kf_fa_fwd_jvp": (ctypes.c_int, [_c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr,
                                     _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, ctypes.c_float,
                                     ctypes.c_int, ctypes.c_int, _c_ptr]),
    "kf_fa_bwd_workspace_size": (ctypes.c_size_t, [_c_i64, _c_i64, _c_i64, _c_i64, ctypes.c_int]),
    "kf_fa_bwd": (ctypes.c_int, [_c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr,
                                 ctypes.c_size_t, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, ctypes.c_float,
                                 ctypes.c_int, ctypes.c_int, ctypes.c_int, _c_ptr]),
}


def _load():
    if not LIB_PATH.exists():
        raise ImportError(
            f"kernelforge_b200 CUDA library not found at {LIB_PATH}; build it with "
            "`python -m kernelforge_b200.build` (nvcc with sm_100a support is required)"
        )
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    return lib


lib = _load()


def status_string(code: int) -> str:
    return lib.kf_status_string(code).decode()


def check(code: int, what: str) -> None:
    if code != KF_OK:
        raise RuntimeError(f"{what} failed: {status_string(code)} (kf_status {code})")


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return DTYPE_CODES[dtype]
    except KeyError:
        raise ValueError(f"unsupported dtype {dtype}; expected float32, float16 or bfloat16") from None


def query_device_error(device=None) -> int:
    """Synchronise and return the first kernel-reported failure (0 when none)."""
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    code = ctypes.c_int(0)
    with torch.cuda.device(device):
        check(lib.kf_query_device_error(stream_handle(device), ctypes.byref(code)), "kf_query_device_error")
    return code.value


def require_cuda(t: torch.Tensor, name: str) -> None:
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
