"""SANA LiteLA attention modules over this library's linear-attention kernel.

Drop-ins for the module API of SANA_LinearAttention/custom.py:391-959 and the package exports of
SANA_LinearAttention/__init__.py:3-27:

* ``LiteLA`` -- the attention block of original.py:66-145, with the constructor of either form
  (original.py:71-82, or custom.py:394-410 with keyword ``batch``, ``seq_len``, ``dtype``).
  Parameters keep the reference's names and shapes: ``qkv`` = Linear(C, 3C, bias=use_bias),
  ``proj`` = Linear(C, C), and ``q_norm`` / ``k_norm`` RMSNorm weights when ``qk_norm``. Reference
  state dicts load unchanged.
* ``JointLiteLA`` (custom.py:526-605), ``CustomOpJointLiteLA`` (custom.py:885-921, one opaque
  ``torch.library`` op for torch.compile), ``CUDAGraphJointLiteLA`` (custom.py:923-959),
  ``GroupedFull64QOutLiteLA`` (custom.py:812-862, its fixed shape) and ``optimized_joint_litela``
  (custom.py:864-870).
* ``qkv_projection`` (custom.py:83-85): ``x [B, N, C] @ WeightT [C, 3C]``.

The attention runs on ``kf_sana_linattn_fwd`` (``qkv_attn_matmul``); both projections run on
this library's tcgen05 GEMM (``kf_linear_fwd``, ``projection.linear``), with the output
projection's bias (and the QKV bias, with ``use_bias``) added in its epilogue. The modules are
inference modules, as the reference's custom ones are: no autograd through the kernels.
``qk_norm`` runs inside the attention kernels (``kf_sana_linattn_qknorm_fwd``: per-token norm
statistics, then q and k normalised as the kernels read them); with rotary embeddings, which
come after the norm, q and k are normalised by this library's RMSNorm kernel first. The
reference's custom modules reject qk_norm.
``apply_rotary_emb`` restates original.py:14-63. With ``rotary_emb`` the modules rotate q and k in
the reference's ``[B, h, d, N]`` layout (SANA's ``use_real_unbind_dim=-2``) and repack them for the
attention kernel.
"""

from __future__ import annotations

import torch

from ..rmsnorm import RMSNorm
from .custom import TORCH_DTYPES, QKVAttnMatmul
from .projection import linear, linear_t, proj_attention

__all__ = [
    "apply_rotary_emb",
    "CUDAGraphJointLiteLA",
    "CustomLiteLA",
    "CustomOpJointLiteLA",
    "GroupedFull64QOutLiteLA",
    "JointLiteLA",
    "LiteLA",
    "optimized_joint_litela",
    "qkv_projection",
]


def qkv_projection(batch: int, seq_len: int, channels: int, dtype: str = "bfloat16"):
    """Return ``project(x, weight_t)``: the no-bias packed QKV projection ``x @ weight_t`` for
    ``x [batch, seq_len, channels]`` and ``weight_t [channels, 3 channels]`` (custom.py:83-85)."""
    if min(batch, seq_len, channels) <= 0:
        raise ValueError("batch, seq_len and channels must be positive")
    torch_dtype = {"float": torch.float32, "float32": torch.float32, "float16": torch.float16,
                   "bfloat16": torch.bfloat16}.get(dtype)
    if torch_dtype is None:
        raise ValueError("dtype must be float, float16, or bfloat16")

    def project(x: torch.Tensor, weight_t: torch.Tensor) -> torch.Tensor:
        if tuple(x.shape) != (batch, seq_len, channels) or tuple(weight_t.shape) != (channels, 3 * channels):
            raise ValueError(f"expected x {(batch, seq_len, channels)} and weight_t {(channels, 3 * channels)}, "
                             f"got {tuple(x.shape)} and {tuple(weight_t.shape)}")
        if x.dtype != torch_dtype or weight_t.dtype != torch_dtype:
            raise ValueError(f"x and weight_t must be {torch_dtype}")
        return linear_t(x, weight_t)

    return project


def apply_rotary_emb(x: torch.Tensor, freqs_cis, use_real: bool = True, use_real_unbind_dim: int = -1) -> torch.Tensor:
    """Rotary position embedding of ``x`` (original.py:14-63).

    ``use_real``: ``freqs_cis = (cos, sin)``, each ``[S, D]``. Element pairs (2i, 2i+1) of the
    head dim become ``(a cos - b sin, b cos + a sin)``: along the last axis of ``[B, H, S, D]``
    (``use_real_unbind_dim=-1``), or along axis -2 of SANA's ``[B, H, D, S]`` with ``cos``/``sin``
    transposed (``-2``). Computed in fp32, returned in ``x``'s dtype. Otherwise ``freqs_cis`` is a
    complex ``[S, D/2]`` tensor multiplying ``x [B, S, H, D]`` viewed as complex pairs.
    """
    if not use_real:
        pairs = torch.view_as_complex(x.float().reshape(*x.shape[:-1], -1, 2))
        return torch.view_as_real(pairs * freqs_cis.unsqueeze(2)).flatten(3).type_as(x)
    cos, sin = (f[None, None].to(x.device) for f in freqs_cis)
    if use_real_unbind_dim == -1:
        a, b = x.reshape(*x.shape[:-1], -1, 2).unbind(-1)
        rotated = torch.stack([-b, a], dim=-1).flatten(3)
    elif use_real_unbind_dim == -2:
        cos, sin = cos.transpose(-1, -2), sin.transpose(-1, -2)
        a, b = x.reshape(*x.shape[:-2], -1, 2, x.shape[-1]).unbind(-2)
        rotated = torch.stack([-b, a], dim=-2).flatten(2, 3)
    else:
        raise ValueError(f"`use_real_unbind_dim={use_real_unbind_dim}` but should be -1 or -2.")
    return (x.float() * cos + rotated.float() * sin).to(x.dtype)


class LiteLA(torch.nn.Module):
    """Lightweight (ReLU) linear attention block (original.py:66-145) on this library's kernel.

    ``batch``, ``seq_len`` and ``dtype`` (keyword) fix the input shape and dtype, as the
    reference's custom module does (custom.py:394-440). Without them any ``[B, N, C]`` input of a
    16-bit or fp32 dtype is accepted, and a kernel is built per shape.
    """

    PAD_VAL = 1  # the ones row of original.py:104, carried as the kernel's ksum row

    def __init__(self, in_dim: int, out_dim: int, heads=None, heads_ratio: float = 1.0, dim: int = 32,
                 eps: float = 1e-15, use_bias: bool = False, qk_norm: bool = False, norm_eps: float = 1e-5, *,
                 batch: int | None = None, seq_len: int | None = None, dtype: torch.dtype | None = None):
        super().__init__()
        heads = heads or int(out_dim // dim * heads_ratio)
        if in_dim % heads != 0 or in_dim % (out_dim // heads) != 0:
            raise ValueError("in_dim must be divisible by the number of heads and by the head dim")
        if dtype is not None and dtype not in TORCH_DTYPES:
            raise ValueError(f"unsupported attention dtype: {dtype}")
        self.in_dim, self.out_dim, self.heads = in_dim, out_dim, heads
        self.dim = out_dim // heads
        self.eps = eps
        self.qkv = torch.nn.Linear(in_dim, 3 * in_dim, bias=use_bias)
        self.proj = torch.nn.Linear(in_dim, in_dim)
        self.kernel_func = torch.nn.ReLU(inplace=False)
        self.qk_norm = qk_norm
        if qk_norm:
            self.q_norm = RMSNorm(in_dim, scale_factor=1.0, eps=norm_eps)
            self.k_norm = RMSNorm(in_dim, scale_factor=1.0, eps=norm_eps)
        else:
            self.q_norm = torch.nn.Identity()
            self.k_norm = torch.nn.Identity()
        self.input_shape = (batch, seq_len, in_dim) if batch is not None and seq_len is not None else None
        self.dtype = dtype
        self._kernels = {}

    def _validate_input(self, x: torch.Tensor) -> None:
        if self.input_shape is not None and tuple(x.shape) != self.input_shape:
            raise ValueError(f"expected LiteLA input shape {self.input_shape}, got {tuple(x.shape)}")
        if self.dtype is not None and x.dtype != self.dtype:
            raise ValueError(f"expected LiteLA dtype {self.dtype}, got {x.dtype}")
        if x.dim() != 3 or x.shape[-1] != self.in_dim:
            raise ValueError(f"expected a [B, N, {self.in_dim}] input, got {tuple(x.shape)}")

    def _attention_kernel(self, batch: int, seq_len: int, dtype: torch.dtype) -> QKVAttnMatmul:
        key = (batch, seq_len, dtype)
        kernel = self._kernels.get(key)
        if kernel is None:
            # The packed QKV holds in_dim / dim heads of `dim` channels (original.py:130-132).
            name = TORCH_DTYPES[dtype]
            kernel = QKVAttnMatmul(batch, self.in_dim // self.dim, self.dim, seq_len, self.eps, name, name)
            self._kernels[key] = kernel
        return kernel

    def _project_qkv(self, x: torch.Tensor) -> torch.Tensor:
        return linear(x, self.qkv.weight, self.qkv.bias)

    def _project_output(self, out: torch.Tensor) -> torch.Tensor:
        return linear(out, self.proj.weight, self.proj.bias)

    def _normalise_qk(self, qkv: torch.Tensor) -> torch.Tensor:
        """q_norm / k_norm over the channels of the packed q and k slices (original.py:127-128)."""
        if not self.qk_norm:
            return qkv
        qkv = qkv.clone()
        qkv[:, :, 0] = self.q_norm(qkv[:, :, 0])
        qkv[:, :, 1] = self.k_norm(qkv[:, :, 1])
        return qkv

    def _attend(self, qkv: torch.Tensor, rotary_emb) -> torch.Tensor:
        """qk_norm (when set), rotary embedding (when given) and attention of a packed qkv. Without
        rotary embedding the norm runs inside the attention kernels (no normalised copy)."""
        if (self.qk_norm and rotary_emb is None and not getattr(self, "fp32_attention", False)
                and self.q_norm.weight.dtype == qkv.dtype and self.k_norm.weight.dtype == qkv.dtype
                and self.q_norm.eps == self.k_norm.eps):
            kernel = self._attention_kernel(qkv.shape[0], qkv.shape[1], qkv.dtype)
            return kernel.with_qk_norm(qkv, self.q_norm.weight, self.k_norm.weight, self.q_norm.eps)
        return self.attention(self._rotate_qk(self._normalise_qk(qkv), rotary_emb))

    def attention(self, qkv: torch.Tensor) -> torch.Tensor:
        """Packed ``[B, N, 3, C]`` QKV -> ``[B, N, C]`` in QKV's dtype (original.py:99-117)."""
        batch, seq_len = qkv.shape[0], qkv.shape[1]
        if getattr(self, "fp32_attention", False):
            out = self._attention_kernel(batch, seq_len, torch.float32)(qkv.float())
            return out.to(qkv.dtype)
        return self._attention_kernel(batch, seq_len, qkv.dtype)(qkv)

    def _rotate_qk(self, qkv: torch.Tensor, rotary_emb) -> torch.Tensor:
        """Rotary embedding of q and k in the reference's [B, h, d, N] layout (original.py:133-135),
        repacked into [B, N, 3, C] for the attention kernel."""
        if rotary_emb is None:
            return qkv
        batch, seq_len, _, channels = qkv.shape
        heads = channels // self.dim

        def rotate(t):  # [B, N, C] -> [B, h, d, N] -> rotated -> [B, N, C]
            hdn = t.transpose(1, 2).reshape(batch, heads, self.dim, seq_len)
            out = apply_rotary_emb(hdn, rotary_emb, use_real_unbind_dim=-2)
            return out.reshape(batch, channels, seq_len).transpose(1, 2)

        return torch.stack([rotate(qkv[:, :, 0]), rotate(qkv[:, :, 1]), qkv[:, :, 2]], dim=2).contiguous()

    def forward(self, x, mask=None, HW=None, rotary_emb=None, block_id=None, block_mask=None):
        self._validate_input(x)
        batch, seq_len, channels = x.shape
        qkv = self._project_qkv(x).reshape(batch, seq_len, 3, channels)
        return self._project_output(self._attend(qkv, rotary_emb))


# The reference's custom module (custom.py:391) is exported as CustomLiteLA next to the original.
CustomLiteLA = LiteLA


class JointLiteLA(LiteLA):
    """LiteLA with the packed QKV projection, attention and bias-fused output projection as three
    launches (custom.py:526-605). ``batch``, ``seq_len`` and ``dtype`` are required; ``in_dim``
    must equal ``out_dim``."""

    def __init__(self, in_dim: int, out_dim: int, *, batch: int, seq_len: int, dtype: torch.dtype, heads=None,
                 heads_ratio: float = 1.0, dim: int = 32, eps: float = 1e-15, use_bias: bool = False,
                 qk_norm: bool = False, norm_eps: float = 1e-5):
        if in_dim != out_dim:
            raise ValueError("JointLiteLA requires in_dim == out_dim")
        super().__init__(in_dim, out_dim, heads, heads_ratio, dim, eps, use_bias, qk_norm, norm_eps, batch=batch,
                         seq_len=seq_len, dtype=dtype)

    # Packed transposed weights under the reference's buffer names (custom.py:437-440, 560-573),
    # as views of the parameters, so they never go stale.
    @property
    def qkv_weight_t(self) -> torch.Tensor:
        return self.qkv.weight.t()

    @property
    def proj_weight_t(self) -> torch.Tensor:
        return self.proj.weight.t()

    @property
    def proj_bias(self) -> torch.Tensor:
        return self.proj.bias

    def forward(self, x, mask=None, HW=None, rotary_emb=None, block_id=None, block_mask=None):
        self._validate_input(x)
        batch, seq_len, channels = x.shape
        qkv = self._project_qkv(x).reshape(batch, seq_len, 3, channels)
        return self._project_output(self._attend(qkv, rotary_emb))


GROUPED_SHAPE = dict(batch=1, seq_len=1024, channels=1152, heads=36, dim=32)


class GroupedFull64QOutLiteLA(JointLiteLA):
    """The reference's fixed-shape specialisation (custom.py:812-862): B=1, N=1024, C=1152, H=36,
    D=32, bf16, no qk_norm and no bias. Like the reference's grouped kernels, its attention never
    writes q, k or v: the QKV projection and the attention run as two fused launches
    (``projection.proj_attention``, ``kf_sana_proj_attn_fwd``, which are not tied to this shape),
    then the bias-fused output projection. The constructor keeps the reference's shape contract."""

    def grouped_attention(self, x: torch.Tensor) -> torch.Tensor:
        """QKV projection + attention without materialising q, k, v (custom.py:851-853)."""
        return proj_attention(x, self.qkv.weight, self.qkv.bias, self.eps)

    def __init__(self, *args, **kwargs):
        in_dim = args[0] if args else kwargs.get("in_dim")
        out_dim = args[1] if len(args) > 1 else kwargs.get("out_dim")
        heads = kwargs.get("heads")
        g = GROUPED_SHAPE
        if ((kwargs.get("batch"), kwargs.get("seq_len"), in_dim, out_dim) != (g["batch"], g["seq_len"], g["channels"],
                                                                               g["channels"])
                or (heads is not None and heads != g["heads"]) or kwargs.get("dtype") != torch.bfloat16
                or kwargs.get("dim", g["dim"]) != g["dim"] or kwargs.get("qk_norm", False)
                or kwargs.get("use_bias", False)):
            raise ValueError("GroupedFull64QOutLiteLA requires exactly B=1,N=1024,C=1152,H=36,D=32, "
                             "bf16, qk_norm=False, and use_bias=False")
        super().__init__(*args, **kwargs)

    def forward(self, x, mask=None, HW=None, rotary_emb=None, block_id=None, block_mask=None):
        if rotary_emb is not None:
            raise ValueError("GroupedFull64QOutLiteLA requires rotary_emb=None")
        self._validate_input(x)
        if getattr(self, "fp32_attention", False):
            return super().forward(x, mask, HW, None, block_id, block_mask)
        return self._project_output(self.grouped_attention(x))


def optimized_joint_litela(in_dim: int, out_dim: int, **kwargs):
    """The module the reference picks for a shape (custom.py:864-870)."""
    shape = (kwargs.get("batch"), kwargs.get("seq_len"), in_dim)
    g = GROUPED_SHAPE
    cls = GroupedFull64QOutLiteLA if shape == (g["batch"], g["seq_len"], g["channels"]) else JointLiteLA
    return cls(in_dim, out_dim, **kwargs)


_PIPELINES: dict = {}


def _pipeline(batch: int, seq_len: int, heads: int, dim: int, eps: float, dtype: torch.dtype) -> QKVAttnMatmul:
    key = (batch, seq_len, heads, dim, float(eps), dtype)
    kernel = _PIPELINES.get(key)
    if kernel is None:
        name = TORCH_DTYPES[dtype]
        kernel = QKVAttnMatmul(batch, heads, dim, seq_len, eps, name, name)
        _PIPELINES[key] = kernel
    return kernel


@torch.library.custom_op("kernelforge_b200::joint_litela_forward", mutates_args=(), device_types="cuda")
def _joint_litela_forward(x: torch.Tensor, qkv_weight_t: torch.Tensor, proj_weight_t: torch.Tensor,
                          proj_bias: torch.Tensor, heads: int, dim: int, eps: float) -> torch.Tensor:
    """QKV projection, attention and output projection as one opaque operator (custom.py:885-898)."""
    batch, seq_len, channels = x.shape
    qkv = linear_t(x, qkv_weight_t).reshape(batch, seq_len, 3, channels)
    out = _pipeline(batch, seq_len, heads, dim, eps, x.dtype)(qkv)
    return linear_t(out, proj_weight_t, proj_bias)


@_joint_litela_forward.register_fake
def _joint_litela_forward_fake(x, qkv_weight_t, proj_weight_t, proj_bias, heads, dim, eps):
    return x.new_empty((*x.shape[:-1], proj_weight_t.shape[-1]))


class CustomOpJointLiteLA(JointLiteLA):
    """JointLiteLA exposed to torch.compile as one opaque operator (custom.py:905-921)."""

    def forward(self, x, mask=None, HW=None, rotary_emb=None, block_id=None, block_mask=None):
        if rotary_emb is not None or self.qk_norm or getattr(self, "fp32_attention", False):
            return super().forward(x, mask, HW, rotary_emb, block_id, block_mask)
        if self.qkv.bias is not None:  # the operator has no QKV bias: the three-launch path adds it
            return super().forward(x, mask, HW, rotary_emb, block_id, block_mask)
        self._validate_input(x)
        return _joint_litela_forward(x, self.qkv_weight_t, self.proj_weight_t, self.proj_bias, self.heads,
                                     self.dim, self.eps)


class CUDAGraphJointLiteLA:
    """Fixed-shape CUDA-graph replay of a JointLiteLA, the input copy included (custom.py:923-959)."""

    def __init__(self, module: JointLiteLA):
        self.module = module
        self.static_input = torch.empty(module.input_shape, device=module.proj.weight.device, dtype=module.dtype)
        warmup_stream = torch.cuda.Stream()
        warmup_stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(warmup_stream), torch.inference_mode():
            for _ in range(3):  # builds the kernels and their workspaces outside the capture
                module(self.static_input)
        torch.cuda.current_stream().wait_stream(warmup_stream)
        self.graph = torch.cuda.CUDAGraph()
        with torch.inference_mode(), torch.cuda.graph(self.graph):
            self.static_output = module(self.static_input)

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        self.static_input.copy_(x)
        self.graph.replay()
        return self.static_output
