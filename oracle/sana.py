"""CPU oracle for SANA ReLU linear attention -- TEST INFRASTRUCTURE ONLY.

Restates ``LiteLA.attn_matmul`` (SANA_LinearAttention/original.py:99-117) and the packed-QKV
views that the reference harness feeds it (SANA_LinearAttention/test.py:52-57, 74-75):

    q, k = ReLU(q), ReLU(k)                      # q, v: [B, h, d, N]; k: [B, h, N, d]
    v'   = [v ; 1]                               # one padding row of ones  -> [B, h, d+1, N]
    vk   = v' @ k                                # [B, h, d+1, d], rounded to the input dtype
    o    = (vk @ q).float()                      # [B, h, d+1, N]
    out  = o[:, :, :d] / (o[:, :, d:] + eps)     # fp32

``attn_matmul_reference`` keeps the reference's intermediate roundings (low-precision
matmul outputs); ``attn_exact`` evaluates the same formula in float64 without intermediate
rounding, which is what the CUDA kernel's fp32 accumulation approximates.
"""

from __future__ import annotations

import torch


def unpack_qkv(qkv: torch.Tensor, heads: int, dim: int):
    """Packed ``[B, N, 3, C]`` -> the (q, k, v) views of SANA test.py:54-57."""
    batch, seq_len, three, channels = qkv.shape
    assert three == 3 and channels == heads * dim
    q, k, v = qkv.unbind(2)
    q = q.transpose(-1, -2).reshape(batch, heads, dim, seq_len)
    k = k.transpose(-1, -2).reshape(batch, heads, dim, seq_len).transpose(-1, -2)
    v = v.transpose(-1, -2).reshape(batch, heads, dim, seq_len)
    return q, k, v


def heads_to_tokens(out: torch.Tensor) -> torch.Tensor:
    """``[B, h, d, N]`` -> ``[B, N, h*d]`` (SANA test.py:74-75 / original.py:142)."""
    batch, heads, dim, seq_len = out.shape
    return out.reshape(batch, heads * dim, seq_len).permute(0, 2, 1).contiguous()


def attn_matmul_reference(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, eps: float = 1e-15):
    """Reference-semantics ``attn_matmul`` on the CPU; returns fp32 ``[B, h, d, N]``."""
    q, k, v = (t.detach().cpu() for t in (q, k, v))
    q = torch.clamp_min(q, 0)
    k = torch.clamp_min(k, 0)
    ones = torch.ones(*v.shape[:-2], 1, v.shape[-1], dtype=v.dtype)
    v_aug = torch.cat([v, ones], dim=-2)
    vk = torch.matmul(v_aug, k)
    full = torch.matmul(vk, q)
    if full.dtype in (torch.float16, torch.bfloat16):
        full = full.float()
    numerator, denominator = full[:, :, :-1], full[:, :, -1:]
    return numerator / (denominator + eps)


def qkv_attention_reference(qkv: torch.Tensor, heads: int, dim: int, eps: float = 1e-15):
    """Packed ``[B, N, 3, C]`` -> fp32 ``[B, N, C]`` with reference roundings."""
    return heads_to_tokens(attn_matmul_reference(*unpack_qkv(qkv.detach().cpu(), heads, dim), eps))


def attn_exact(qkv: torch.Tensor, heads: int, dim: int, eps: float = 1e-15) -> torch.Tensor:
    """Float64 evaluation of the same formula: packed ``[B, N, 3, C]`` -> ``[B, N, C]``."""
    x = qkv.detach().to("cpu", torch.float64)
    batch, seq_len, _, channels = x.shape
    q = torch.clamp_min(x[:, :, 0].reshape(batch, seq_len, heads, dim), 0)
    k = torch.clamp_min(x[:, :, 1].reshape(batch, seq_len, heads, dim), 0)
    v = x[:, :, 2].reshape(batch, seq_len, heads, dim)
    vk = torch.einsum("bnhr,bnhc->bhrc", v, k)          # sum over tokens: [B, h, d, d]
    ksum = k.sum(dim=1)                                  # [B, h, d]
    num = torch.einsum("bhrc,bnhc->bnhr", vk, q)
    den = torch.einsum("bhc,bnhc->bnh", ksum, q)[..., None]
    return (num / (den + eps)).reshape(batch, seq_len, channels)


def rmsnorm_exact(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """Float64 RMSNorm over the last axis (rmsnorm/original.py:27-52, without roundings)."""
    x = x.to(torch.float64)
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * weight.to(torch.float64)


def litela_forward_exact(x, qkv_weight, qkv_bias, proj_weight, proj_bias, dim, eps=1e-15,
                         q_norm_weight=None, k_norm_weight=None, norm_eps=1e-5):
    """Float64 ``LiteLA.forward`` (SANA_LinearAttention/original.py:119-145) without rotary
    embeddings: packed QKV projection, optional q / k RMSNorm over the channels, ReLU linear
    attention with the ones-row denominator, output projection. ``x``: ``[B, N, C]``."""
    x = x.detach().to("cpu", torch.float64)
    batch, seq_len, channels = x.shape
    qkv = x @ qkv_weight.detach().to("cpu", torch.float64).t()
    if qkv_bias is not None:
        qkv = qkv + qkv_bias.detach().to("cpu", torch.float64)
    q, k, v = qkv.reshape(batch, seq_len, 3, channels).unbind(2)
    if q_norm_weight is not None:
        q = rmsnorm_exact(q, q_norm_weight.detach().cpu(), norm_eps)
        k = rmsnorm_exact(k, k_norm_weight.detach().cpu(), norm_eps)
    out = attn_exact(torch.stack([q, k, v], dim=2), channels // dim, dim, eps)
    return out @ proj_weight.detach().to("cpu", torch.float64).t() + proj_bias.detach().to("cpu", torch.float64)



def linear_exact(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
    """Float64 ``x @ weight.T + bias`` for an nn.Linear weight ``[out, in]``: the projections of
    ``LiteLA.forward`` (SANA_LinearAttention/original.py:122 ``self.qkv``, :143 ``self.proj``),
    which the reference's TileLang kernels compute with fp32 accumulation
    (SANA_LinearAttention/custom.py:23-85, 457-523). Unrounded: a kernel's fp32 accumulation
    rounded once to a 16-bit dtype lands within one ulp of it."""
    y = x.detach().to("cpu", torch.float64) @ weight.detach().to("cpu", torch.float64).t()
    if bias is not None:
        y = y + bias.detach().to("cpu", torch.float64)
    return y


def qk_inv_rms(qkv: torch.Tensor, eps: float) -> torch.Tensor:
    """Float64 ``1 / sqrt(mean(x^2) + eps)`` of every token's q and k rows of a packed
    ``[B, N, 3, C]`` qkv -> ``[B, N, 2]``: the scale of LiteLA's q_norm / k_norm
    (SANA_LinearAttention/original.py:127-128, RMSNorm._norm of rmsnorm/original.py:27-38)."""
    x = qkv.detach().to("cpu", torch.float64)[:, :, :2]
    return 1.0 / torch.sqrt((x * x).mean(-1) + eps)


def qk_norm_apply(qkv: torch.Tensor, q_weight: torch.Tensor, k_weight: torch.Tensor, inv_rms: torch.Tensor):
    """q_norm / k_norm of a packed qkv with the given per-token scales ``inv_rms [B, N, 2]``
    (fp32 values), with the reference's rounding points (rmsnorm/original.py:51-52): the
    normalised row rounded to the input dtype, then multiplied by the weight and rounded again
    (fp32 inputs: two fp32 multiplies). v is unchanged."""
    q, k, v = qkv.detach().cpu().unbind(2)
    r = inv_rms.detach().cpu().to(torch.float32)
    dtype = qkv.dtype

    def norm(x, rr, w):
        return (x.float() * rr[..., None]).to(dtype) * w.detach().cpu().to(dtype)

    return torch.stack([norm(q, r[..., 0], q_weight), norm(k, r[..., 1], k_weight), v], dim=2)
