"""One-pass RMSNorm (drop-in for the reference's ``rmsnorm`` package, rmsnorm/__init__.py:1-4)."""

from .custom import (RMSNorm, RMSNormFunction, original_tilelang_rms_norm, rms_norm, rmsnorm_backward,
                     rmsnorm_forward, rmsnorm_into)
from .custom import rms_norm as custom_rms_norm

__all__ = ["RMSNorm", "RMSNormFunction", "custom_rms_norm", "original_tilelang_rms_norm", "rms_norm",
           "rmsnorm_backward", "rmsnorm_forward", "rmsnorm_into"]
