"""SANA ReLU linear attention (drop-in for SANA_LinearAttention/__init__.py:3-27)."""

from .custom import QKVAttnMatmul, qkv_attn_matmul, sana_linattn_into
from .modules import (
    CUDAGraphJointLiteLA,
    apply_rotary_emb,
    CustomLiteLA,
    CustomOpJointLiteLA,
    GroupedFull64QOutLiteLA,
    JointLiteLA,
    LiteLA,
    optimized_joint_litela,
    qkv_projection,
)
from .projection import linear, linear_t

__all__ = [
    "apply_rotary_emb",
    "CUDAGraphJointLiteLA",
    "CustomLiteLA",
    "CustomOpJointLiteLA",
    "GroupedFull64QOutLiteLA",
    "JointLiteLA",
    "LiteLA",
    "linear",
    "linear_t",
    "QKVAttnMatmul",
    "optimized_joint_litela",
    "qkv_attn_matmul",
    "qkv_projection",
    "sana_linattn_into",
]
