"""SANA attention fused with its QKV projection (kf_sana_proj_attn_fwd) on the GPU.

The reference's grouped kernels (SANA_LinearAttention/custom.py:595-868) compute LiteLA's QKV
projection and ReLU linear attention without writing q, k or v. Oracle: the float64 attention
(``oracle.sana.attn_exact``) of the packed qkv that this library's projection GEMM writes
(fp32 accumulation rounded to bf16, the rounding the fused kernels apply to K, V and Q), with the
SANA bar (bf16 out within 1 ulp + atol 2e-3), and the unfused path (projection GEMM + attention
kernel) within twice that. Shapes: the reference's own (1, 1024, 1152), token counts that are not
multiples of the 128-token tile, a last head group with fewer than 4 heads (70 heads), a single
partial group (3 heads), with and without the QKV bias.
"""

import pytest
import torch

from oracle import sana as oracle
from tests.tolerances import assert_close_ulp_atol

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def proj():
    if not torch.cuda.is_available():
        pytest.skip("CUDA is required")
    from kernelforge_b200.SANA_LinearAttention import projection

    return projection


@pytest.mark.parametrize("bias", [False, True])
@pytest.mark.parametrize("b,n,c", [(1, 1024, 1152), (2, 1000, 256), (1, 300, 2240), (3, 77, 96)])
def test_fused_projection_attention(proj, b, n, c, bias):
    from kernelforge_b200.SANA_LinearAttention import QKVAttnMatmul

    g = torch.Generator().manual_seed(b * 1000 + n + c + bias)
    x = torch.randn(b, n, c, generator=g).to(torch.bfloat16).cuda()
    w = (torch.randn(3 * c, c, generator=g) / c ** 0.5).to(torch.bfloat16).cuda()
    bb = (0.1 * torch.randn(3 * c, generator=g)).to(torch.bfloat16).cuda() if bias else None
    out = proj.proj_attention(x, w, bb)
    assert out.shape == (b, n, c) and out.dtype == torch.bfloat16
    qkv = proj.linear(x, w, bb).view(b, n, 3, c)
    heads = c // 32
    expected = oracle.attn_exact(qkv.cpu(), heads, 32)
    assert_close_ulp_atol(out, expected, dtype=torch.bfloat16, ulps=1, atol=2e-3)
    unfused = QKVAttnMatmul(b, heads, 32, n, 1e-15, "bfloat16", "bfloat16")(qkv)
    assert_close_ulp_atol(out, unfused.double().cpu(), dtype=torch.bfloat16, ulps=2, atol=4e-3)
    assert torch.equal(proj.proj_attention(x, w, bb), out)  # deterministic


def test_fused_projection_attention_rejects_unsupported(proj):
    from kernelforge_b200 import _lib

    x = torch.zeros(1, 64, 64, dtype=torch.float16, device="cuda")
    w = torch.zeros(192, 64, dtype=torch.float16, device="cuda")
    with pytest.raises(RuntimeError, match="unsupported"):
        proj.proj_attention(x, w)
    with pytest.raises(ValueError):
        proj.proj_attention(x.bfloat16(), w[:100].bfloat16())
    assert _lib.query_device_error() == 0
