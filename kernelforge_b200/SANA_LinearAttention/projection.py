"""SANA's projection GEMMs on the sm_100a tensor cores (``kf_linear_fwd``).

``linear(x, weight, bias)`` is ``torch.nn.functional.linear`` for a ``[..., in]`` input and an
nn.Linear weight ``[out, in]``; ``linear_t(x, weight_t, bias)`` takes the reference's prepacked
``WeightT [in, out]`` (SANA_LinearAttention/custom.py:23-85 ``_qkv_projection`` and :457-523
``_output_projection``). Either weight may also be passed as the transposed view of the other
layout: the call reads whichever layout is dense in memory, so no transpose is copied.
fp16/bf16 run the tcgen05 kernel (fp32 accumulation, bias added in fp32, one rounding); fp32
runs fp32 FMAs.
"""

from __future__ import annotations

import torch

from .. import _lib

_KN = 1  # weight_layout: [in, out]
_NK = 0  # weight_layout: [out, in] (nn.Linear)


def _dense_weight(w_nk: torch.Tensor):
    """(tensor, layout) for a logical [out, in] weight, without copying when either layout is dense."""
    if w_nk.is_contiguous():
        return w_nk, _NK
    if w_nk.t().is_contiguous():
        return w_nk.t(), _KN
    return w_nk.contiguous(), _NK


def _project(x: torch.Tensor, w_nk: torch.Tensor, bias: torch.Tensor | None) -> torch.Tensor:
    _lib.require_cuda(x, "x")
    out_features, in_features = w_nk.shape
    if x.shape[-1] != in_features:
        raise ValueError(f"x has {x.shape[-1]} features, the weight expects {in_features}")
    if w_nk.dtype != x.dtype or w_nk.device != x.device:
        raise ValueError("the weight must have x's dtype and device")
    if bias is not None and (bias.shape != (out_features,) or bias.dtype != x.dtype or bias.device != x.device):
        raise ValueError(f"bias must be a [{out_features}] tensor with x's dtype and device")
    weight, layout = _dense_weight(w_nk)
    rows = x.reshape(-1, in_features) if x.is_contiguous() else x.contiguous().reshape(-1, in_features)
    bias = None if bias is None else bias.contiguous()
    y = torch.empty((*x.shape[:-1], out_features), dtype=x.dtype, device=x.device)
    with torch.cuda.device(x.device):
        status = _lib.lib.kf_linear_fwd(rows.data_ptr(), weight.data_ptr(), None if bias is None else bias.data_ptr(),
                                        y.data_ptr(), rows.shape[0], in_features, out_features, layout,
                                        _lib.dtype_code(x.dtype), _lib.stream_handle(x.device))
    _lib.check(status, "kf_linear_fwd")
    return y


def linear(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
    """``x @ weight.T + bias`` for an nn.Linear weight ``[out, in]``."""
    return _project(x, weight, bias)


def linear_t(x: torch.Tensor, weight_t: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
    """``x @ weight_t + bias`` for a prepacked ``weight_t [in, out]``."""
    return _project(x, weight_t.t(), bias)


def proj_attention(x: torch.Tensor, qkv_weight: torch.Tensor, qkv_bias: torch.Tensor | None = None,
                   eps: float = 1e-15) -> torch.Tensor:
    """LiteLA's QKV projection and linear attention in two launches that never write q, k or v
    (``kf_sana_proj_attn_fwd``): ``x [B, N, C]`` and the packed nn.Linear weight
    ``qkv_weight [3C, C]`` (bias ``[3C]`` or None) -> the attention output ``[B, N, C]`` in x's
    dtype, before the output projection. Heads of 32 channels; bf16 (as the reference's grouped
    kernels)."""
    _lib.require_cuda(x, "x")
    if x.dim() != 3:
        raise ValueError("x must be [batch, seq_len, channels]")
    batch, seq_len, channels = x.shape
    if tuple(qkv_weight.shape) != (3 * channels, channels) or qkv_weight.dtype != x.dtype:
        raise ValueError(f"qkv_weight must be a [{3 * channels}, {channels}] tensor of x's dtype")
    if qkv_bias is not None and (tuple(qkv_bias.shape) != (3 * channels,) or qkv_bias.dtype != x.dtype):
        raise ValueError(f"qkv_bias must be a [{3 * channels}] tensor of x's dtype")
    x = x.contiguous()
    weight = qkv_weight.contiguous()
    bias = None if qkv_bias is None else qkv_bias.contiguous()
    ws_bytes = _lib.lib.kf_sana_proj_attn_workspace_size(batch, seq_len, channels)
    if ws_bytes == 0:
        raise ValueError("channels must be a positive multiple of 32")
    workspace = torch.empty(ws_bytes, dtype=torch.uint8, device=x.device)
    out = torch.empty_like(x)
    with torch.cuda.device(x.device):
        status = _lib.lib.kf_sana_proj_attn_fwd(x.data_ptr(), weight.data_ptr(), None if bias is None else bias.data_ptr(),
                                                out.data_ptr(), workspace.data_ptr(), ws_bytes, batch, seq_len,
                                                channels, float(eps), _lib.dtype_code(x.dtype),
                                                _lib.stream_handle(x.device))
    _lib.check(status, "kf_sana_proj_attn_fwd")
    return out
