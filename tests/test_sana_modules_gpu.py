"""SANA LiteLA modules on the GPU against the float64 module oracle.

Mirrors the reference harness's end-to-end check (SANA_LinearAttention/test.py:106-155): the
joint module, its custom-op form under torch.compile and its CUDA-graph wrapper, each loaded from
one state dict, against the original module's math, with the harness tolerance rtol = atol = 2e-2
(atol scaled by the output's magnitude). Oracle: ``oracle.sana.litela_forward_exact``.
"""

import pytest
import torch

from oracle import sana as oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def sana():
    if not torch.cuda.is_available():
        pytest.skip("CUDA is required")
    import kernelforge_b200.SANA_LinearAttention as mod

    return mod


def expected(module, x, norm=False):
    return oracle.litela_forward_exact(
        x, module.qkv.weight, module.qkv.bias, module.proj.weight, module.proj.bias, module.dim, module.eps,
        module.q_norm.weight if norm else None, module.k_norm.weight if norm else None,
        module.q_norm.eps if norm else 1e-5)


def assert_close(actual, ref):
    scale = max(1.0, ref.abs().max().item())
    torch.testing.assert_close(actual.detach().cpu().double(), ref, rtol=2e-2, atol=2e-2 * scale)


def build(sana, cls, b, n, c, dtype, seed=0, **kw):
    torch.manual_seed(seed)
    return cls(c, c, batch=b, seq_len=n, dtype=dtype, heads=c // 32, dim=32, **kw).cuda().to(dtype).eval()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("b,n,c", [(2, 512, 256), (1, 1000, 1152), (4, 4096, 1152)])
def test_joint_custom_op_and_graph_match_the_oracle(sana, b, n, c, dtype):
    joint = build(sana, sana.JointLiteLA, b, n, c, dtype)
    custom = build(sana, sana.CustomOpJointLiteLA, b, n, c, dtype, seed=1)
    custom.load_state_dict(joint.state_dict())
    x = torch.randn(b, n, c, device="cuda", dtype=dtype)
    ref = expected(joint, x)
    with torch.inference_mode():
        direct = joint(x).clone()
        op = custom(x).clone()
        graph = sana.CUDAGraphJointLiteLA(joint)
        replayed = graph(x).clone()
    assert direct.shape == (b, n, c) and direct.dtype == dtype
    for out in (direct, op, replayed):
        assert_close(out, ref)
    torch.testing.assert_close(replayed, direct, rtol=1e-2, atol=1e-2)  # same kernels, same inputs


def test_custom_op_under_torch_compile(sana):
    b, n, c, dtype = 1, 1024, 256, torch.bfloat16
    custom = build(sana, sana.CustomOpJointLiteLA, b, n, c, dtype)
    compiled = torch.compile(custom, fullgraph=True)
    x = torch.randn(b, n, c, device="cuda", dtype=dtype)
    with torch.inference_mode():
        eager = custom(x).clone()
        traced = compiled(x).clone()
    torch.testing.assert_close(traced, eager, rtol=0, atol=0)


def test_grouped_shape_module(sana):
    m = build(sana, sana.GroupedFull64QOutLiteLA, 1, 1024, 1152, torch.bfloat16)
    x = torch.randn(1, 1024, 1152, device="cuda", dtype=torch.bfloat16)
    with torch.inference_mode():
        assert_close(m(x), expected(m, x))
    with pytest.raises(ValueError, match="rotary_emb"):
        m(x, rotary_emb=(torch.zeros(1), torch.zeros(1)))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_litela_any_shape_qk_norm_and_bias(sana, dtype):
    torch.manual_seed(3)
    m = sana.LiteLA(128, 128, heads=4, dim=32, use_bias=True, qk_norm=True).cuda().to(dtype).eval()
    with torch.no_grad():
        m.q_norm.weight.uniform_(0.5, 1.5)
        m.k_norm.weight.uniform_(0.5, 1.5)
    for b, n in ((1, 300), (3, 77)):
        x = torch.randn(b, n, 128, device="cuda", dtype=dtype)
        with torch.inference_mode():
            assert_close(m(x), expected(m, x, norm=True))


def test_fp32_attention_flag(sana):
    m = build(sana, sana.JointLiteLA, 2, 256, 256, torch.bfloat16)
    m.fp32_attention = True
    x = torch.randn(2, 256, 256, device="cuda", dtype=torch.bfloat16)
    with torch.inference_mode():
        assert_close(m(x), expected(m, x))


@pytest.mark.parametrize("index", range(3))
def test_reference_module_fixtures(sana, index):
    """The reference's own LiteLA.forward (original.py:119-145; qk_norm, bias, rotary embeddings)
    on fp32 inputs, its state dict loaded into this library's module (tests/golden)."""
    from pathlib import Path

    case = torch.load(Path(__file__).resolve().parent / "golden" / "sana_modules_golden.pt")["modules"][index]
    b, n, c = case["x"].shape
    m = sana.LiteLA(c, c, heads=case["heads"], dim=case["dim"], qk_norm=case["qk_norm"],
                    use_bias=case["use_bias"]).cuda().eval()
    m.load_state_dict(case["state"])
    rot = tuple(t.cuda() for t in case["rotary"]) if case["rotary"] is not None else None
    with torch.inference_mode():
        out = m(case["x"].cuda(), rotary_emb=rot)
    torch.testing.assert_close(out.cpu(), case["out"], rtol=1e-3, atol=1e-4)
