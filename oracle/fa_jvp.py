"""CPU oracle for attention, its LSE and its forward-mode JVP -- TEST INFRASTRUCTURE ONLY.

Restates the dense references of flash_attention_jvp/original.py:

* ``attention``                  (original.py:6-30)  dense softmax attention, GQA, bottom-right
  aligned causal mask, rows with no valid key return zero;
* ``attention_jvp``              (original.py:33-39) ``torch.func.jvp`` of ``attention``;
* ``attention_jvp_from_forward`` (original.py:42-65) the standalone JVP from cached O and LSE:
  ``tO = P tV + H V - rowsum(H) * O`` with ``P = exp(gamma S - LSE)`` and
  ``H = P * gamma (tQ K^T + Q tK^T)``;
* ``attention_lse``  natural-log LSE ``[B, Hq, Nq]`` with ``+inf`` for rows without a valid
  key, the convention that the reference kernel documents for FlashAttention's LSE
  (flash_attention_jvp/custom.py:70-72).

Tensors use the reference layout ``[B, S, H, D]``. Low-precision inputs are evaluated with
fp32 intermediates and cast back; float64 inputs stay float64.
"""

from __future__ import annotations

import torch


def _scale(q, softmax_scale):
    return q.shape[-1] ** -0.5 if softmax_scale is None else float(softmax_scale)


def _heads_first(x, dtype, groups=1):
    x = x.to(dtype).transpose(1, 2)
    return x.repeat_interleave(groups, dim=1) if groups > 1 else x


def causal_valid(nq: int, nk: int, device=None) -> torch.Tensor:
    """Bottom-right aligned causal mask: key j is visible to query i iff j <= i + nk - nq."""
    rows = torch.arange(nq, device=device)[:, None]
    cols = torch.arange(nk, device=device)[None, :]
    return cols <= rows + (nk - nq)


def attention(q, k, v, *, softmax_scale=None, causal=False):
    dtype = torch.float64 if q.dtype == torch.float64 else torch.float32
    groups = q.shape[2] // k.shape[2]
    qh = _heads_first(q, dtype)
    kh = _heads_first(k, dtype, groups)
    vh = _heads_first(v, dtype, groups)
    logits = torch.matmul(qh, kh.transpose(-1, -2)) * _scale(q, softmax_scale)
    if causal:
        valid = causal_valid(q.shape[1], k.shape[1], q.device)
        logits = logits.masked_fill(~valid, float("-inf"))
        # A query row with no visible key would be NaN after softmax; FlashAttention
        # returns zeros there, so give it finite logits and zero its weights below.
        logits = torch.where(valid.any(dim=-1, keepdim=True), logits, torch.zeros_like(logits))
    weights = torch.softmax(logits, dim=-1)
    if causal:
        weights = weights.masked_fill(~valid, 0.0)
    return torch.matmul(weights, vh).transpose(1, 2).to(q.dtype)


def attention_jvp(q, k, v, tq, tk, tv, *, softmax_scale=None, causal=False):
    """Return ``(out, tangent)`` by differentiating ``attention`` with ``torch.func.jvp``."""
    primals = (q, k, v)
    tangents = tuple(torch.zeros_like(p) if t is None else t for p, t in zip(primals, (tq, tk, tv)))
    return torch.func.jvp(
        lambda a, b, c: attention(a, b, c, softmax_scale=softmax_scale, causal=causal),
        primals,
        tangents,
    )


def attention_lse(q, k, *, softmax_scale=None, causal=False):
    """Natural-log LSE ``[B, Hq, Nq]`` (float32 unless the inputs are float64)."""
    dtype = torch.float64 if q.dtype == torch.float64 else torch.float32
    groups = q.shape[2] // k.shape[2]
    qh = _heads_first(q, dtype)
    kh = _heads_first(k, dtype, groups)
    logits = torch.matmul(qh, kh.transpose(-1, -2)) * _scale(q, softmax_scale)
    if causal:
        valid = causal_valid(q.shape[1], k.shape[1], q.device)
        logits = logits.masked_fill(~valid, float("-inf"))
    lse = torch.logsumexp(logits, dim=-1)
    # logsumexp of an all -inf row is -inf; FlashAttention reports +inf for empty rows.
    return torch.where(torch.isneginf(lse), torch.full_like(lse, float("inf")), lse)


@torch.no_grad()
def attention_jvp_from_forward(q, k, v, tq, tk, tv, out, lse, *, softmax_scale=None, causal=False):
    """Standalone dense JVP that reuses a cached ``out`` and natural-log ``lse``."""
    primals = (q, k, v)
    tangents = tuple(torch.zeros_like(p) if t is None else t for p, t in zip(primals, (tq, tk, tv)))
    groups = q.shape[2] // k.shape[2]
    qh, tqh = (_heads_first(x, torch.float32) for x in (q, tangents[0]))
    kh, vh, tkh, tvh = (_heads_first(x, torch.float32, groups) for x in (k, v, tangents[1], tangents[2]))
    scale = _scale(q, softmax_scale)
    weights = torch.exp(torch.matmul(qh, kh.transpose(-1, -2)) * scale - lse.float()[..., None])
    if causal:
        valid = causal_valid(q.shape[1], k.shape[1], q.device)
        weights = weights.masked_fill(~valid, 0.0)
    dlogits = (torch.matmul(tqh, kh.transpose(-1, -2)) + torch.matmul(qh, tkh.transpose(-1, -2))) * scale
    h = weights * dlogits
    result = torch.matmul(weights, tvh) + torch.matmul(h, vh) - h.sum(-1, keepdim=True) * out.float().transpose(1, 2)
    return result.transpose(1, 2).to(q.dtype)
