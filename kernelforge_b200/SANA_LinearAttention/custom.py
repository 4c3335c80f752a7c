"""SANA ReLU linear attention on the sm_100a kernels (``kf_sana_linattn_fwd``).

Drop-in for the reference's ``qkv_attn_matmul`` (SANA_LinearAttention/custom.py:340-388):

    run = qkv_attn_matmul(batch, heads, dim, seq_len, eps=1e-15, dtype="bfloat16",
                          output_dtype="float", reduce_splits=True)
    out = run(qkv)       # qkv [batch, seq_len, 3, heads*dim] -> out [batch, seq_len, heads*dim]

computing ``LiteLA.attn_matmul`` (SANA_LinearAttention/original.py:99-117) on the packed
layout with fp32 accumulation of K^T V and sum(ReLU(K)).
"""

from __future__ import annotations

import torch

from .. import _lib

THREADS = 128
TORCH_DTYPES = {torch.float16: "float16", torch.bfloat16: "bfloat16", torch.float32: "float"}


class QKVAttnMatmul:
    """Callable returned by :func:`qkv_attn_matmul`.

    It owns a device workspace (fp32 split partials, the reduced K^T V / sum(ReLU(K)) and one
    arrival counter per head group), allocated zero-filled on first use per device and reused
    by every later call, so the callable is CUDA-graph capturable after its first call.
    Calls through one callable must be ordered on one stream (they share the workspace).
    ``splits``: None or 0 picks the schedule automatically, -1 forces the one-launch path
    (whole heads per CTA, or per thread-block cluster when there are fewer heads than SMs; no
    workspace traffic), a positive count the split path with that many token chunks
    (``kf_sana_linattn_fwd`` in include/kernelforge_b200.h). :meth:`plan` reports the choice.
    """

    def __init__(self, batch, heads, dim, seq_len, eps, dtype, output_dtype, splits=None):
        self.batch, self.heads, self.dim, self.seq_len = batch, heads, dim, seq_len
        self.eps = float(eps)
        self.dtype = _lib.DTYPE_NAMES[dtype]
        self.output_dtype = _lib.DTYPE_NAMES[output_dtype]
        self.splits = int(splits) if splits else 0
        # Sized for the qk_norm form too (the same layout plus the per-token norm statistics), so
        # one workspace serves both entry points.
        self.workspace_bytes = _lib.lib.kf_sana_linattn_qknorm_workspace_size(batch, heads, dim, seq_len,
                                                                               self.splits)
        if self.workspace_bytes == 0:
            raise ValueError("unsupported SANA attention shape")
        self._workspaces = {}

    def workspace(self, device: torch.device) -> torch.Tensor:
        ws = self._workspaces.get(device)
        if ws is None:
            ws = torch.zeros(self.workspace_bytes, dtype=torch.uint8, device=device)
            self._workspaces[device] = ws
        return ws

    def plan(self, device=None) -> tuple[int, int]:
        """(kernel launches per call, CTAs per (batch, head) unit on the one-launch path or 0)
        for this shape on ``device`` (default: the current CUDA device), without launching."""
        import ctypes

        launches, ctas = ctypes.c_int64(0), ctypes.c_int64(0)
        device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        with torch.cuda.device(device):
            status = _lib.lib.kf_sana_linattn_plan(self.batch, self.heads, self.dim, self.seq_len, self.splits,
                                                   _lib.dtype_code(self.dtype), ctypes.byref(launches),
                                                   ctypes.byref(ctas))
        _lib.check(status, "kf_sana_linattn_plan")
        return launches.value, ctas.value

    def __call__(self, qkv: torch.Tensor) -> torch.Tensor:
        expected = (self.batch, self.seq_len, 3, self.heads * self.dim)
        if tuple(qkv.shape) != expected:
            raise ValueError(f"qkv must have shape {expected}, got {tuple(qkv.shape)}")
        if qkv.dtype != self.dtype:
            raise ValueError(f"qkv must be {self.dtype}, got {qkv.dtype}")
        _lib.require_cuda(qkv, "qkv")
        qkv = qkv.contiguous()
        out = torch.empty((self.batch, self.seq_len, self.heads * self.dim), dtype=self.output_dtype,
                          device=qkv.device)
        return sana_linattn_into(qkv, out, self.workspace(qkv.device), self.heads, self.dim,
                                 self.eps, self.splits)


    def with_qk_norm(self, qkv: torch.Tensor, q_weight: torch.Tensor, k_weight: torch.Tensor,
                     norm_eps: float) -> torch.Tensor:
        """The attention of ``qkv`` after LiteLA's qk_norm (SANA_LinearAttention/original.py:127-128):
        q and k each through an RMSNorm over their token's channels with ``q_weight`` /
        ``k_weight`` (``[heads * dim]``, qkv's dtype) and ``norm_eps``, applied inside the
        attention kernels as they read q and k (``kf_sana_linattn_qknorm_fwd``); qkv is not
        modified and no normalised copy is made."""
        expected = (self.batch, self.seq_len, 3, self.heads * self.dim)
        if tuple(qkv.shape) != expected or qkv.dtype != self.dtype:
            raise ValueError(f"qkv must be a {expected} {self.dtype} tensor")
        channels = self.heads * self.dim
        for name, w in (("q_weight", q_weight), ("k_weight", k_weight)):
            if w.shape != (channels,) or w.dtype != qkv.dtype or w.device != qkv.device:
                raise ValueError(f"{name} must be a [{channels}] tensor with qkv's dtype and device")
        qkv = qkv.contiguous()
        out = torch.empty((self.batch, self.seq_len, channels), dtype=self.output_dtype, device=qkv.device)
        ws = self.workspace(qkv.device)
        q_weight, k_weight = q_weight.contiguous(), k_weight.contiguous()
        with torch.cuda.device(qkv.device):
            status = _lib.lib.kf_sana_linattn_qknorm_fwd(
                qkv.data_ptr(), out.data_ptr(), ws.data_ptr(), ws.numel(), self.batch, self.heads, self.dim,
                self.seq_len, self.splits, self.eps, q_weight.data_ptr(), k_weight.data_ptr(), float(norm_eps),
                _lib.dtype_code(qkv.dtype), _lib.dtype_code(out.dtype), _lib.stream_handle(qkv.device))
        _lib.check(status, "kf_sana_linattn_qknorm_fwd")
        return out


def sana_linattn_into(qkv, out, workspace, heads, dim, eps, splits=0):
    """Launch ``kf_sana_linattn_fwd`` on the current stream of ``qkv``'s device."""
    batch, seq_len = qkv.shape[0], qkv.shape[1]
    with torch.cuda.device(qkv.device):
        status = _lib.lib.kf_sana_linattn_fwd(
            qkv.data_ptr(), out.data_ptr(), workspace.data_ptr(), workspace.numel(),
            batch, heads, dim, seq_len, int(splits or 0), float(eps),
            _lib.dtype_code(qkv.dtype), _lib.dtype_code(out.dtype), _lib.stream_handle(qkv.device),
        )
    _lib.check(status, "kf_sana_linattn_fwd")
    return out


def qkv_attn_matmul(
    batch: int,
    heads: int,
    dim: int,
    seq_len: int,
    eps: float = 1e-15,
    dtype: str = "bfloat16",
    output_dtype: str = "float",
    reduce_splits: bool = True,
):
    """Return ``run(qkv)`` for packed ``[batch, seq_len, 3, heads*dim]`` QKV.

    ``reduce_splits`` selected between two partial-reduction kernels in the reference; here the
    K^T V partials are always summed once, in a fixed order (in shared memory on the one-launch
    path, while building the epilogue's B operand on the split path), so the flag is accepted
    for signature compatibility and does not change the result.
    """
    if dim <= 0 or dim > THREADS or THREADS % dim != 0:
        raise ValueError(f"dim must divide {THREADS} and be at most {THREADS}")
    if output_dtype not in ("float", "float16", "bfloat16"):
        raise ValueError("output_dtype must be float, float16, or bfloat16")
    if dtype not in ("float", "float16", "bfloat16"):
        raise ValueError("dtype must be float, float16, or bfloat16")
    if min(batch, heads, seq_len) <= 0:
        raise ValueError("batch, heads and seq_len must be positive")
    del reduce_splits
    return QKVAttnMatmul(int(batch), int(heads), int(dim), int(seq_len), eps, dtype, output_dtype)
