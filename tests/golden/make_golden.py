"""Generate the golden fixtures under tests/golden/ by running the REFERENCE itself.

This script imports the reference's own framework-native baselines (the three ``original.py``
files of zzd1992/KernelForge) from a checkout of the reference and runs them on the CPU on
small, seeded inputs. It writes ``*.pt`` fixtures holding the inputs and the reference's
outputs. The fixtures are committed; the tests never need the reference checkout.

Usage:  python tests/golden/make_golden.py /path/to/KernelForge [rmsnorm sana sana_modules fa_jvp]

``SANA_LinearAttention/original.py`` imports ``timm`` only for the ``Attention`` base class
of ``LiteLA`` (original.py:10, 65, 83); ``timm`` is not installed here, so a stub base class
that creates the ``qkv``/``proj`` linear layers is registered before the import. The
function under test, ``LiteLA.attn_matmul`` (original.py:99-117), touches only
``self.kernel_func`` and ``self.eps``, so the stub does not change its arithmetic. The module
fixtures run ``LiteLA.forward`` (original.py:119-145), which uses only the base class's
``qkv = Linear(C, 3C, bias=qkv_bias)`` and ``proj = Linear(C, C)``, the layers the stub creates
as timm's ``Attention`` does.
"""

from __future__ import annotations

import sys
import types
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent


def _install_timm_stub():
    if "timm" in sys.modules:
        return

    class Attention(torch.nn.Module):
        def __init__(self, dim, num_heads=8, qkv_bias=False, **_):
            super().__init__()
            self.num_heads = num_heads
            self.qkv = torch.nn.Linear(dim, dim * 3, bias=qkv_bias)
            self.proj = torch.nn.Linear(dim, dim)

    timm = types.ModuleType("timm")
    models = types.ModuleType("timm.models")
    vit = types.ModuleType("timm.models.vision_transformer")
    vit.Attention = Attention
    timm.models = models
    models.vision_transformer = vit
    sys.modules.update({"timm": timm, "timm.models": models, "timm.models.vision_transformer": vit})


def _gen(seed):
    g = torch.Generator().manual_seed(seed)
    return g


def make_rmsnorm(ref_root: Path):
    from rmsnorm.original import RMSNorm  # noqa: E402  (reference module)

    cases = []
    # (shape, dtype, eps): odd dims and non-multiple-of-8 widths exercise the ragged paths.
    specs = [
        ((2, 3, 1000), torch.bfloat16, 1e-6),
        ((1, 4, 4096), torch.bfloat16, 1e-6),
        ((3, 7, 256), torch.float16, 1e-6),
        ((2, 5, 77), torch.float32, 1e-6),
        ((1, 2, 8192), torch.bfloat16, 1e-5),
        ((4, 1, 130), torch.bfloat16, 1e-6),
    ]
    for i, (shape, dtype, eps) in enumerate(specs):
        g = _gen(100 + i)
        x = torch.randn(shape, generator=g).to(dtype)
        w = (1.0 + 0.1 * torch.randn(shape[-1], generator=g)).to(dtype)
        module = RMSNorm(shape[-1], eps=eps).to(dtype)
        module.weight.data.copy_(w)
        with torch.no_grad():
            y = module(x)
        cases.append(dict(x=x, weight=w, eps=eps, y=y))
    torch.save(cases, HERE / "rmsnorm_golden.pt")
    return len(cases)


def make_sana(ref_root: Path):
    _install_timm_stub()
    from SANA_LinearAttention.original import LiteLA  # noqa: E402  (reference module)

    cases = []
    # (batch, seq_len, heads, dim, dtype)
    specs = [
        (1, 100, 2, 32, torch.bfloat16),
        (2, 257, 3, 32, torch.bfloat16),
        (1, 64, 2, 32, torch.float16),
        (1, 50, 2, 32, torch.float32),
        (1, 96, 2, 16, torch.bfloat16),
        (1, 40, 1, 64, torch.float32),
    ]
    for i, (batch, seq_len, heads, dim, dtype) in enumerate(specs):
        g = _gen(200 + i)
        channels = heads * dim
        qkv = torch.randn(batch, seq_len, 3, channels, generator=g).to(dtype)
        q, k, v = qkv.unbind(2)
        q = q.transpose(-1, -2).reshape(batch, heads, dim, seq_len)
        k = k.transpose(-1, -2).reshape(batch, heads, dim, seq_len).transpose(-1, -2)
        v = v.transpose(-1, -2).reshape(batch, heads, dim, seq_len)
        module = LiteLA(channels, channels, heads=heads, dim=dim, qk_norm=False).to(dtype).eval()
        with torch.no_grad():
            out = module.attn_matmul(q, k, v)
        out = out.view(batch, channels, seq_len).permute(0, 2, 1).contiguous()
        cases.append(dict(qkv=qkv, heads=heads, dim=dim, eps=module.eps, out=out))
    torch.save(cases, HERE / "sana_golden.pt")
    return len(cases)


def make_sana_modules(ref_root: Path):
    """``apply_rotary_emb`` (original.py:14-63) and a full ``LiteLA.forward`` (original.py:119-145)
    with qk_norm and rotary embeddings, from the reference's own module."""
    _install_timm_stub()
    from SANA_LinearAttention.original import LiteLA, apply_rotary_emb  # noqa: E402  (reference)

    g = _gen(300)
    rotary = []
    for dtype in (torch.float32, torch.bfloat16):
        x = torch.randn(2, 3, 10, 8, generator=g).to(dtype)          # [B, H, S, D]
        cos, sin = torch.randn(10, 8, generator=g), torch.randn(10, 8, generator=g)
        rotary.append(dict(x=x, cos=cos, sin=sin, dim=-1, out=apply_rotary_emb(x, (cos, sin), True, -1)))
        xt = torch.randn(2, 3, 8, 10, generator=g).to(dtype)         # [B, H, D, S] (SANA)
        rotary.append(dict(x=xt, cos=cos, sin=sin, dim=-2, out=apply_rotary_emb(xt, (cos, sin), True, -2)))
    xc = torch.randn(2, 10, 3, 8, generator=g)                        # [B, S, H, D], complex form
    freqs = torch.polar(torch.ones(1, 10, 4), torch.randn(1, 10, 4, generator=g))  # [1, S, D/2]
    rotary.append(dict(x=xc, freqs=freqs, out=apply_rotary_emb(xc, freqs, use_real=False)))

    modules = []
    # (batch, seq_len, channels, heads, qk_norm, use_bias, rotary)
    for i, (b, n, c, h, qk_norm, bias, use_rot) in enumerate([(2, 77, 128, 4, True, True, True),
                                                            (1, 130, 64, 2, False, False, True),
                                                            (1, 64, 96, 3, True, False, False)]):
        gm = _gen(310 + i)
        torch.manual_seed(310 + i)
        module = LiteLA(c, c, heads=h, dim=c // h, qk_norm=qk_norm, use_bias=bias).eval()
        if qk_norm:
            with torch.no_grad():
                module.q_norm.weight.uniform_(0.5, 1.5)
                module.k_norm.weight.uniform_(0.5, 1.5)
        x = torch.randn(b, n, c, generator=gm)
        rot = (torch.randn(n, c // h, generator=gm), torch.randn(n, c // h, generator=gm)) if use_rot else None
        with torch.no_grad():
            out = module(x, rotary_emb=rot)
        modules.append(dict(x=x, rotary=rot, heads=h, dim=c // h, qk_norm=qk_norm, use_bias=bias,
                            state=module.state_dict(), out=out))
    torch.save(dict(rotary=rotary, modules=modules), HERE / "sana_modules_golden.pt")
    return len(rotary) + len(modules)


def make_fa(ref_root: Path):
    from flash_attention_jvp.original import attention, attention_jvp, attention_jvp_from_forward

    cases = []
    # B, Nq, Nk, Hq, Hkv, D, causal, scale -- a subset of flash_attention_jvp/test.py:25-38.
    specs = [
        (1, 7, 11, 2, 2, 8, False, None),
        (2, 33, 65, 4, 4, 24, False, 0.3),
        (1, 65, 65, 2, 2, 64, True, None),
        (1, 19, 71, 4, 2, 96, True, None),
        (1, 71, 19, 4, 1, 32, True, None),
        (1, 9, 13, 2, 1, 256, False, None),
        (1, 1, 1, 2, 2, 64, True, None),
    ]
    for i, (b, nq, nk, h, hk, d, causal, scale) in enumerate(specs):
        g = _gen(300 + i)
        shapes = ((b, nq, h, d), (b, nk, hk, d), (b, nk, hk, d))
        # Values exactly representable in both bf16 and fp16, so a GPU test can run the same
        # fixture in either dtype; the reference runs them in float64.
        prim = [_half_exact(torch.randn(s, generator=g)) for s in shapes]
        tang = [_half_exact(torch.randn(s, generator=g)) for s in shapes]
        out, tangent = attention_jvp(*prim, *tang, softmax_scale=scale, causal=causal)
        # LSE for the standalone form, in float32 as FlashAttention returns it.
        lse = _lse64(prim[0], prim[1], scale, causal).float()
        dense = attention_jvp_from_forward(
            *(x.float() for x in prim), *(x.float() for x in tang), out.float(), lse,
            softmax_scale=scale, causal=causal,
        )
        small = {name: t.to(torch.bfloat16) for name, t in zip(("q", "k", "v", "tq", "tk", "tv"), (*prim, *tang))}
        cases.append(dict(case=(b, nq, nk, h, hk, d, causal, scale), **small,
                          out=out.float(), tangent=tangent.float(), lse=lse,
                          dense_from_forward=dense, attention_out_fp32=attention(
                              *(x.float() for x in prim), softmax_scale=scale, causal=causal)))
    torch.save(cases, HERE / "fa_jvp_golden.pt")
    return len(cases)


def _half_exact(x):
    """Round to bf16, flush values below fp16's normal range, return float64."""
    x = x.to(torch.bfloat16).double()
    return torch.where(x.abs() < 2.0 ** -14, torch.zeros_like(x), x)


def _lse64(q, k, scale, causal):
    groups = q.shape[2] // k.shape[2]
    qh = q.transpose(1, 2)
    kh = k.transpose(1, 2).repeat_interleave(groups, dim=1)
    s = (qh @ kh.transpose(-1, -2)) * (q.shape[-1] ** -0.5 if scale is None else scale)
    if causal:
        nq, nk = q.shape[1], k.shape[1]
        valid = torch.arange(nk)[None, :] <= torch.arange(nq)[:, None] + nk - nq
        s = s.masked_fill(~valid, float("-inf"))
    lse = torch.logsumexp(s, dim=-1)
    return torch.where(torch.isneginf(lse), torch.full_like(lse, float("inf")), lse)


def main():
    if len(sys.argv) < 2:
        raise SystemExit(__doc__)
    ref_root = Path(sys.argv[1]).resolve()
    parts = sys.argv[2:] or ["rmsnorm", "sana", "sana_modules", "fa_jvp"]
    sys.path.insert(0, str(ref_root))
    torch.set_num_threads(4)
    makers = {"rmsnorm": make_rmsnorm, "sana": make_sana, "sana_modules": make_sana_modules, "fa_jvp": make_fa}
    for part in parts:
        print(f"{part} cases:", makers[part](ref_root))


if __name__ == "__main__":
    main()
