"""SANA LiteLA module API without a GPU: construction, parameter layout (reference state dicts
load unchanged), shape contracts and validation (SANA_LinearAttention/custom.py:391-959)."""

import pytest
import torch

from kernelforge_b200 import SANA_LinearAttention as sana


def test_state_dict_keys_match_the_reference_layout():
    m = sana.JointLiteLA(256, 256, batch=2, seq_len=64, dtype=torch.bfloat16, heads=8, dim=32)
    assert sorted(m.state_dict()) == ["proj.bias", "proj.weight", "qkv.weight"]
    assert m.qkv.weight.shape == (768, 256) and m.proj.weight.shape == (256, 256)
    biased = sana.LiteLA(256, 256, use_bias=True, qk_norm=True)
    assert sorted(biased.state_dict()) == ["k_norm.weight", "proj.bias", "proj.weight", "q_norm.weight",
                                           "qkv.bias", "qkv.weight"]
    # Loading one module's state into another keeps the transposed-weight views in step.
    other = sana.JointLiteLA(256, 256, batch=2, seq_len=64, dtype=torch.bfloat16, heads=8, dim=32)
    other.load_state_dict(m.state_dict())
    assert torch.equal(other.qkv_weight_t, m.qkv.weight.t()) and torch.equal(other.proj_bias, m.proj.bias)


def test_shape_contracts_and_validation():
    with pytest.raises(ValueError, match="in_dim == out_dim"):
        sana.JointLiteLA(256, 512, batch=1, seq_len=64, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="requires exactly"):
        sana.GroupedFull64QOutLiteLA(1152, 1152, batch=2, seq_len=1024, dtype=torch.bfloat16, heads=36, dim=32)
    with pytest.raises(ValueError, match="unsupported attention dtype"):
        sana.LiteLA(64, 64, dtype=torch.int8)
    m = sana.JointLiteLA(64, 64, batch=1, seq_len=32, dtype=torch.bfloat16, heads=2, dim=32)
    with pytest.raises(ValueError, match="input shape"):
        m(torch.zeros(1, 16, 64, dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="CUDA"):  # the attention kernel needs a GPU tensor
        sana.LiteLA(64, 64)(torch.zeros(1, 8, 64))
    project = sana.qkv_projection(1, 8, 64, "bfloat16")
    with pytest.raises(ValueError, match="weight_t"):
        project(torch.zeros(1, 8, 64, dtype=torch.bfloat16), torch.zeros(64, 64, dtype=torch.bfloat16))


def test_optimized_joint_litela_picks_the_reference_module():
    kwargs = dict(dtype=torch.bfloat16, heads=36, dim=32)
    grouped = sana.optimized_joint_litela(1152, 1152, batch=1, seq_len=1024, **kwargs)
    joint = sana.optimized_joint_litela(1152, 1152, batch=2, seq_len=1024, **kwargs)
    assert type(grouped) is sana.GroupedFull64QOutLiteLA and type(joint) is sana.JointLiteLA
    assert sana.CustomLiteLA is sana.LiteLA


GOLDEN = __import__("pathlib").Path(__file__).resolve().parent / "golden" / "sana_modules_golden.pt"


def test_apply_rotary_emb_matches_the_reference_fixtures():
    """Fixtures from the reference's own apply_rotary_emb (original.py:14-63), all three forms."""
    cases = torch.load(GOLDEN)["rotary"]
    for case in cases:
        if "freqs" in case:
            out = sana.apply_rotary_emb(case["x"], case["freqs"], use_real=False)
        else:
            out = sana.apply_rotary_emb(case["x"], (case["cos"], case["sin"]), True, case["dim"])
        assert out.dtype == case["out"].dtype
        torch.testing.assert_close(out, case["out"], rtol=0, atol=0)
