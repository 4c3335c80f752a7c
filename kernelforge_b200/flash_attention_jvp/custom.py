"""FlashAttention forward, forward-mode JVP and backward on the sm_100a kernels (``kf_fa_*``).

Public names and call signatures are the reference's (flash_attention_jvp/custom.py and its
``__init__``): ``flash_attention``, ``flash_attention_jvp``, ``get_jvp_config``,
``FlashAttentionFunction``, ``_attention_jvp_kernel``, plus the module attributes its harness
touches (``_flash_attn_forward``, which test.py:75 patches to prove that the standalone JVP
runs no forward, and ``_flash_attn_backward``). Validation raises ``ValueError`` with the
fragments the harness matches ("lse", "tq", "finite", "positive", "float16", "pipeline").

How this module is organised:

* ``Problem`` describes one call (sizes, softmax scale) and is built by ``_problem``, the one
  place where q, k, v and the scale are checked. The C ABI re-checks the same domain and
  answers with a status code, so a call that reaches a kernel has passed both.
* ``JvpSchedule`` holds the reference's tile/pipeline arguments. The reference compiles a
  kernel per schedule; the kernels here pick their own tiles, so a schedule is validated over
  the reference's domain, resolved to the same defaults ``get_jvp_config`` reports, and has no
  effect on the result. Forward and JVP results are deterministic for a given shape; the
  backward is too with ``deterministic=True`` (otherwise dq may vary in its last bit).
* Every kernel is wrapped in an opaque ``torch.library`` operator (``kernelforge_b200::…``), so
  torch.func transforms unwrap their tensors before a raw pointer is taken, and fake kernels
  give shapes to tracing.
* ``FlashAttentionFunction`` ties the forward operator to two rules: the reverse-mode rule runs
  the backward operator, the forward-mode rule runs the standalone JVP operator on the saved O
  and LSE (no second forward).

Differences from the reference, by design:

* the forward (O and the natural-log LSE) is this library's kernel, not the flash_attn binary,
  so ``flash_attention`` matches ``flash_attn_func`` within tolerance, not bitwise;
* ``flash_attention_fwd_jvp`` adds the one-pass forward + JVP (O, LSE and tO from one scan over
  the keys, flash-attention-jvp-derivation.md sections 7-8);
* a ``None`` tangent reaches the kernel as a null pointer and its GEMM is skipped (the
  reference materialises zeros); the result is the same.
"""

from __future__ import annotations

import math
from typing import NamedTuple, Optional

import torch
from torch.autograd.function import once_differentiable

from .. import _lib

_OP_NAMESPACE = "kernelforge_b200"
_INPUT_DTYPES = (torch.float16, torch.bfloat16)
_MAX_HEAD_DIM = 256


# ---------------------------------------------------------------------------------------------
# the call: sizes and scale, checked once (domain of flash_attention_jvp/custom.py:160-177)
# ---------------------------------------------------------------------------------------------
class Problem(NamedTuple):
    """Sizes and softmax scale of one attention call (q [B, Nq, Hq, D], k/v [B, Nk, Hkv, D])."""

    batch: int
    q_len: int
    k_len: int
    q_heads: int
    kv_heads: int
    head_dim: int
    scale: float

    @property
    def lse_shape(self):
        return (self.batch, self.q_heads, self.q_len)


def _problem(q, k, v, softmax_scale) -> Problem:
    """Check q, k, v and the scale against what the kernels support; raise ``ValueError``."""
    if not all(t.ndim == 4 for t in (q, k, v)):
        raise ValueError("q, k and v must be 4-D tensors laid out [batch, sequence, heads, dim]")
    if q.dtype not in _INPUT_DTYPES:
        raise ValueError(f"inputs must be float16 or bfloat16 tensors, not {q.dtype}")
    if not q.is_cuda or {k.device, v.device} != {q.device} or {k.dtype, v.dtype} != {q.dtype}:
        raise ValueError("q, k and v must live on one CUDA device and share one dtype")
    batch, q_len, q_heads, head_dim = q.shape
    k_len, kv_heads = k.shape[1], k.shape[2]
    if min(batch, q_len, k_len, q_heads, kv_heads, head_dim) < 1:
        raise ValueError("every size (batch, both sequence lengths, heads, head dim) must be positive")
    if v.shape != k.shape or k.shape[0] != batch or k.shape[3] != head_dim:
        raise ValueError("k and v need equal shapes, with q's batch size and head dim")
    if q_heads % kv_heads or head_dim % 8 or head_dim > _MAX_HEAD_DIM:
        raise ValueError(f"unsupported heads/dim: q heads ({q_heads}) must be a multiple of kv heads "
                         f"({kv_heads}); head dim ({head_dim}) a multiple of 8, at most {_MAX_HEAD_DIM}")
    scale = float(softmax_scale) if softmax_scale is not None else 1.0 / math.sqrt(head_dim)
    if not (math.isfinite(scale) and scale > 0.0):
        raise ValueError(f"softmax_scale must be finite and positive (got {scale})")
    return Problem(batch, q_len, k_len, q_heads, kv_heads, head_dim, scale)


def _validate_inputs(q, k, v, softmax_scale):
    """The reference's validation entry point: checks the call and returns its softmax scale."""
    return _problem(q, k, v, softmax_scale).scale


def _check_saved_forward(problem: Problem, q, out, lse):
    if out.shape != q.shape or out.dtype != q.dtype or out.device != q.device:
        raise ValueError("out must be the forward output: q's shape, dtype and device")
    if tuple(lse.shape) != problem.lse_shape or lse.dtype != torch.float32 or lse.device != q.device:
        raise ValueError(f"lse must be the forward's float32 {list(problem.lse_shape)} tensor on q's device")


def _prepare_tangent(tangent, primal, name):
    """A tangent as the kernel takes it: dense, or ``None`` for a zero tangent."""
    if tangent is None:
        return None
    if (tangent.shape, tangent.dtype, tangent.device) != (primal.shape, primal.dtype, primal.device):
        raise ValueError(f"{name} must match its primal's shape, dtype and device")
    return tangent.contiguous()


# ---------------------------------------------------------------------------------------------
# the reference's schedule arguments (flash_attention_jvp/custom.py:123-134, 202-217)
# ---------------------------------------------------------------------------------------------
def _pipeline_depth(k_len: int, block_n: int, causal: bool) -> int:
    """One stage when a single key tile covers the scan, or for long non-causal scans; else two."""
    if k_len <= block_n:
        return 1
    return 1 if (k_len >= 8192 and not causal) else 2


class JvpSchedule(NamedTuple):
    """Tile and pipeline arguments in the reference's domain. Validated, reported, not used."""

    block_m: int
    block_n: int
    threads: int
    num_stages: int

    # (block_n, threads) of the reference's recorded defaults, by head-dim class.
    _NARROW = (64, 128)   # head dim <= 128
    _WIDE = (32, 256)     # head dim 136-256

    @classmethod
    def default(cls, head_dim: int, k_len: int, causal: bool) -> "JvpSchedule":
        block_n, threads = cls._WIDE if head_dim > 128 else cls._NARROW
        return cls(64, block_n, threads, _pipeline_depth(k_len, block_n, causal))

    @classmethod
    def resolve(cls, problem: Problem, causal: bool, block_m, block_n, threads, num_stages) -> "JvpSchedule":
        """Explicit arguments win; the rest follow the defaults (16-row tiles default to 128 threads)."""
        base = cls.default(problem.head_dim, problem.k_len, causal)
        bm = base.block_m if block_m is None else block_m
        bn = base.block_n if block_n is None else block_n
        th = threads if threads is not None else (128 if bm == 16 else base.threads)
        st = num_stages if num_stages is not None else _pipeline_depth(problem.k_len, bn, causal)
        return cls(bm, bn, th, st).checked()

    def checked(self) -> "JvpSchedule":
        ok = (self.block_m in (16, 32, 64, 128) and self.block_n in (32, 64, 128)
              and self.threads in (128, 256) and self.num_stages in (1, 2, 3))
        if not ok:
            raise ValueError(f"tile/pipeline arguments {tuple(self)} are outside the supported "
                             "block_m/block_n/threads/num_stages domain")
        return self


def _default_jvp_config(dim, keys, causal):
    """The reference's default schedule for a head dim and key count, as a dict."""
    return JvpSchedule.default(dim, keys, causal)._asdict()


def get_jvp_config(q, k, v, *, softmax_scale=None, causal=False):
    """Default schedule of a call (deterministic; nothing is compiled or tuned)."""
    problem = _problem(q, k, v, softmax_scale)
    return _default_jvp_config(problem.head_dim, problem.k_len, causal)


# ---------------------------------------------------------------------------------------------
# opaque operators around the C ABI
# ---------------------------------------------------------------------------------------------
def _ptr(t):
    return None if t is None else t.data_ptr()


def _abi_call(name, *args):
    """Run a kf_fa_* entry point on the current stream of the first tensor argument's device.

    The C ABI reads every tensor as dense row-major memory from its data pointer, so a strided
    view reaching this point is an error, never a silent misread."""
    tensors = [a for a in args if isinstance(a, torch.Tensor)]
    if not all(t.is_contiguous() for t in tensors):
        raise ValueError(f"{name}: every tensor argument must be contiguous")
    device = tensors[0].device
    raw = [_ptr(a) if isinstance(a, torch.Tensor) or a is None else a for a in args]
    with torch.cuda.device(device):
        status = getattr(_lib.lib, name)(*raw, _lib.stream_handle(device))
    _lib.check(status, name)


def _sizes(q, k):
    return (q.shape[0], q.shape[1], k.shape[1], q.shape[2], k.shape[2], q.shape[3])


def _lse_like(q):
    return q.new_empty((q.shape[0], q.shape[2], q.shape[1]), dtype=torch.float32)


@torch.library.custom_op(f"{_OP_NAMESPACE}::flash_attention_forward", mutates_args=(), device_types="cuda")
def _launch_fwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float, causal: bool
                ) -> tuple[torch.Tensor, torch.Tensor]:
    out, lse = torch.empty_like(q), _lse_like(q)
    _abi_call("kf_fa_fwd", q, k, v, out, lse, *_sizes(q, k), float(scale), int(causal), _lib.dtype_code(q.dtype))
    return out, lse


@_launch_fwd.register_fake
def _(q, k, v, scale, causal):
    return torch.empty_like(q), _lse_like(q)


@torch.library.custom_op(f"{_OP_NAMESPACE}::flash_attention_jvp", mutates_args=(), device_types="cuda")
def _launch_jvp(
    q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
    tq: Optional[torch.Tensor], tk: Optional[torch.Tensor], tv: Optional[torch.Tensor],
    out: torch.Tensor, lse: torch.Tensor,
    scale: float, causal: bool, block_m: int, block_n: int, threads: int, num_stages: int,
) -> torch.Tensor:
    tangent = torch.empty_like(out)
    _abi_call("kf_fa_jvp", q, k, v, tq, tk, tv, out, lse, tangent, *_sizes(q, k), float(scale), int(causal),
              _lib.dtype_code(q.dtype))
    return tangent


@_launch_jvp.register_fake
def _(q, k, v, tq, tk, tv, out, lse, scale, causal, block_m, block_n, threads, num_stages):
    return torch.empty_like(out)


@torch.library.custom_op(f"{_OP_NAMESPACE}::flash_attention_fwd_jvp", mutates_args=(), device_types="cuda")
def _launch_fwd_jvp(
    q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
    tq: Optional[torch.Tensor], tk: Optional[torch.Tensor], tv: Optional[torch.Tensor],
    scale: float, causal: bool,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    out, lse, tangent = torch.empty_like(q), _lse_like(q), torch.empty_like(q)
    _abi_call("kf_fa_fwd_jvp", q, k, v, tq, tk, tv, out, lse, tangent, *_sizes(q, k), float(scale), int(causal),
              _lib.dtype_code(q.dtype))
    return out, lse, tangent


@_launch_fwd_jvp.register_fake
def _(q, k, v, tq, tk, tv, scale, causal):
    return torch.empty_like(q), _lse_like(q), torch.empty_like(q)


def _bwd_into(dout, q, k, v, out, lse, dq, dk, dv, scale, causal, deterministic):
    """kf_fa_bwd into dense gradient buffers (dq like q, dk/dv like k). deterministic=False (what
    the reference passes to flash_attn) runs one kernel whose dQ partials are summed at L2 for
    head dims up to 128; True runs the separate dQ and dK/dV kernels (bitwise reproducible)."""
    flag = int(bool(deterministic))
    ws_bytes = _lib.lib.kf_fa_bwd_workspace_size(q.shape[0], q.shape[2], q.shape[1], q.shape[3], flag)
    workspace = torch.empty(ws_bytes, dtype=torch.uint8, device=q.device)
    _abi_call("kf_fa_bwd", q, k, v, out, dout, lse, dq, dk, dv, workspace, ws_bytes, *_sizes(q, k), float(scale),
              int(bool(causal)), flag, _lib.dtype_code(q.dtype))


@torch.library.custom_op(f"{_OP_NAMESPACE}::flash_attention_backward", mutates_args=(), device_types="cuda")
def _launch_bwd(dout: torch.Tensor, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, out: torch.Tensor,
                lse: torch.Tensor, scale: float, causal: bool, deterministic: bool = False
                ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    _bwd_into(dout, q, k, v, out, lse, dq, dk, dv, scale, causal, deterministic)
    return dq, dk, dv


@_launch_bwd.register_fake
def _(dout, q, k, v, out, lse, scale, causal, deterministic=False):
    return torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)


# ---------------------------------------------------------------------------------------------
# flash_attn-style entry points (the names the reference imports and its harness patches)
# ---------------------------------------------------------------------------------------------
def _plain_attention_only(dropout_p, window_size_left, window_size_right, softcap, alibi_slopes, extra=False):
    if (dropout_p, window_size_left, window_size_right, softcap) != (0.0, -1, -1, 0.0) or alibi_slopes is not None \
            or extra:
        raise NotImplementedError("supported: dropout_p=0, unbounded windows, no softcap, no ALiBi, no returned "
                                  "softmax")


def _flash_attn_forward(q, k, v, dropout_p, softmax_scale, causal, window_size_left=-1,
                        window_size_right=-1, softcap=0.0, alibi_slopes=None, return_softmax=False):
    """This library's forward behind flash_attn's ``_flash_attn_forward`` signature.

    Returns ``(out, lse, None, None)``; lse is fp32 ``[B, Hq, Nq]``, natural log, ``+inf`` for
    a row that sees no key.
    """
    _plain_attention_only(dropout_p, window_size_left, window_size_right, softcap, alibi_slopes, return_softmax)
    out, lse = _launch_fwd(q.contiguous(), k.contiguous(), v.contiguous(), float(softmax_scale), bool(causal))
    return out, lse, None, None


def _flash_attn_backward(dout, q, k, v, out, lse, dq, dk, dv, dropout_p, softmax_scale, causal,
                         window_size_left=-1, window_size_right=-1, softcap=0.0, alibi_slopes=None,
                         deterministic=False):
    """Attention's VJP from the saved O and LSE, behind flash_attn's ``_flash_attn_backward``
    signature: fills dq, dk, dv in place (strided destinations through a dense copy) and returns
    them. ``deterministic`` has flash_attn's meaning: False (the reference's choice) lets dq vary
    in the last bit between runs (its partials are summed at L2); True makes it reproducible."""
    _plain_attention_only(dropout_p, window_size_left, window_size_right, softcap, alibi_slopes)
    dense = [t.contiguous() for t in (dout, q, k, v, out)]
    targets = [g if g.is_contiguous() else torch.empty_like(g, memory_format=torch.contiguous_format)
               for g in (dq, dk, dv)]
    _bwd_into(dense[0], *dense[1:], lse.float().contiguous(), *targets, softmax_scale, causal, deterministic)
    for given, written in zip((dq, dk, dv), targets):
        if given is not written:
            given.copy_(written)
    return dq, dk, dv


# ---------------------------------------------------------------------------------------------
# public API
# ---------------------------------------------------------------------------------------------
def _attention_jvp_kernel(batch, queries, keys, heads, kv_heads, dim, dtype, scale, causal,
                          block_m=64, block_n=64, threads=128, num_stages=2):
    """A callable ``kernel(Q, K, V, TQ, TK, TV, O, LSE) -> TO`` fixed to one shape and dtype."""
    schedule = JvpSchedule(block_m, block_n, threads, num_stages).checked()
    want = {"float16": torch.float16, "bfloat16": torch.bfloat16}[dtype]
    q_shape, kv_shape = (batch, queries, heads, dim), (batch, keys, kv_heads, dim)
    roles = (("Q", q_shape), ("K", kv_shape), ("V", kv_shape), ("TQ", q_shape), ("TK", kv_shape),
             ("TV", kv_shape), ("O", q_shape))

    def kernel(*tensors):
        if len(tensors) != len(roles) + 1:
            raise TypeError(f"kernel takes Q, K, V, TQ, TK, TV, O, LSE; got {len(tensors)} tensors")
        *operands, lse = tensors
        for (name, shape), t in zip(roles, operands):
            if tuple(t.shape) != shape or t.dtype != want:
                raise ValueError(f"{name}: expected {shape} {want}, got {tuple(t.shape)} {t.dtype}")
        return _launch_jvp(*(t.contiguous() for t in operands), lse.contiguous(), float(scale), bool(causal),
                           *schedule)

    return kernel


@torch.no_grad()
def flash_attention_jvp(
    q, k, v, tq, tk, tv, out, lse, *, softmax_scale=None, causal=False,
    block_m=64, block_n=None, threads=None, num_stages=None,
):
    """Tangent of attention's output from the saved forward (O, LSE): no forward launch.

    q/tq: [B, Nq, Hq, D]; k/tk/v/tv: [B, Nk, Hkv, D]; out: [B, Nq, Hq, D]; lse: fp32
    [B, Hq, Nq], natural log, from these primals with this scale and masking. A ``None``
    tangent is zero. Returns a tensor like ``out``.
    """
    problem = _problem(q, k, v, softmax_scale)
    _check_saved_forward(problem, q, out, lse)
    schedule = JvpSchedule.resolve(problem, causal, block_m, block_n, threads, num_stages)
    primals = [t.contiguous() for t in (q, k, v)]
    tangents = [_prepare_tangent(t, p, n) for t, p, n in zip((tq, tk, tv), primals, ("tq", "tk", "tv"))]
    return _launch_jvp(*primals, *tangents, out.contiguous(), lse.contiguous(), problem.scale, bool(causal),
                       *schedule)


@torch.no_grad()
def flash_attention_fwd_jvp(q, k, v, tq, tk, tv, *, softmax_scale=None, causal=False):
    """Forward and tangent in one scan over the keys: returns ``(out, lse, tangent)``.

    Six GEMMs per key tile with online softmax statistics (flash-attention-jvp-derivation.md
    sections 7-8), against 2 + 5 for a forward launch followed by the standalone JVP.
    """
    problem = _problem(q, k, v, softmax_scale)
    primals = [t.contiguous() for t in (q, k, v)]
    tangents = [_prepare_tangent(t, p, n) for t, p, n in zip((tq, tk, tv), primals, ("tq", "tk", "tv"))]
    return _launch_fwd_jvp(*primals, *tangents, problem.scale, bool(causal))


class FlashAttentionFunction(torch.autograd.Function):
    """``(out, lse) = attention(q, k, v)`` with this library's kernels for the value and both
    derivative rules. lse is a non-differentiable by-product, kept so that the forward-mode
    rule can run the standalone JVP on the saved forward instead of a second forward."""

    @staticmethod
    def forward(q, k, v, softmax_scale, causal):
        scale = _problem(q, k, v, softmax_scale).scale
        # Through the module attribute, so a patch of _flash_attn_forward sees every forward.
        out, lse = _flash_attn_forward(q, k, v, 0.0, scale, causal)[:2]
        return out, lse

    @staticmethod
    def setup_context(ctx, inputs, output):
        q, k, v, softmax_scale, causal = inputs
        ctx.scale = _problem(q, k, v, softmax_scale).scale
        ctx.causal = bool(causal)
        saved = (q, k, v, *output)
        ctx.save_for_backward(*saved)
        ctx.save_for_forward(*saved)
        ctx.mark_non_differentiable(output[1])
        ctx.set_materialize_grads(False)

    @staticmethod
    @once_differentiable
    def backward(ctx, grad_out, _grad_lse):
        if grad_out is None:
            return None, None, None, None, None
        q, k, v, out, lse = (t.contiguous() for t in ctx.saved_tensors)
        dq, dk, dv = _launch_bwd(grad_out.contiguous(), q, k, v, out, lse, ctx.scale, ctx.causal)
        return dq, dk, dv, None, None

    @staticmethod
    def jvp(ctx, tq, tk, tv, _t_scale, _t_causal):
        q, k, v, out, lse = (t.contiguous() for t in ctx.saved_tensors)
        schedule = JvpSchedule.default(q.shape[-1], k.shape[1], ctx.causal)
        tangents = [_prepare_tangent(t, p, n) for t, p, n in zip((tq, tk, tv), (q, k, v), ("tq", "tk", "tv"))]
        return _launch_jvp(q, k, v, *tangents, out, lse, ctx.scale, ctx.causal, *schedule), None


def flash_attention(q, k, v, *, softmax_scale=None, causal=False, return_lse=False):
    """Attention with this library's forward, reverse-mode and forward-mode rules.

    Returns ``out``, or ``(out, lse)`` with ``return_lse=True`` (fp32 natural-log LSE, not
    differentiable, the input of a later standalone ``flash_attention_jvp``). Works under
    torch.func.jvp and torch.autograd.forward_ad; first-order derivatives only; no dropout.
    """
    problem = _problem(q, k, v, softmax_scale)
    dense = [t.contiguous() for t in (q, k, v)]
    out, lse = FlashAttentionFunction.apply(*dense, problem.scale, bool(causal))
    return (out, lse) if return_lse else out
