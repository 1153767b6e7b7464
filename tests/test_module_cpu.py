"""Module adapter on CPU: planner-selected exact modes, parameter names, errors.

On a CPU device the planner selects the organiser's exact operation order
(reason unsupported_device), as the reference planner does; the adapter must
then equal BaselineSelfAttention (torch_transformer_benchmark.py:60-123),
restated here from the oracle.
"""

import pytest
import torch
import torch.nn as nn

from b200_attention.attention_dispatch import AttentionMode, AttentionModelSpec, FallbackReason
from b200_attention.modules import B200FusedSelfAttention
from oracle.reference_attention import reference_attention


def baseline_forward(mod: nn.Module, x, mask, causal):
    B, S, d = x.shape
    H = mod.num_heads
    heads = lambda t: t.view(B, S, H, d // H).transpose(1, 2).contiguous()
    ctx = reference_attention(heads(mod.q_proj(x)), heads(mod.k_proj(x)), heads(mod.v_proj(x)),
                              mask, causal, (d // H) ** -0.5)
    out = mod.out_proj(ctx.transpose(1, 2).contiguous().view(B, S, d))
    if mask is not None:
        out = out.masked_fill(~mask[..., None], 0)
    return out


@pytest.mark.parametrize("dtype,mode", [(torch.float32, AttentionMode.FP32_BASELINE_EXACT),
                                        (torch.bfloat16, AttentionMode.EXACT_REFERENCE)])
def test_cpu_exact_mode_equals_baseline(dtype, mode):
    torch.manual_seed(0)
    mod = B200FusedSelfAttention(64, 4).to(dtype).eval()
    x = torch.randn(2, 33, 64).to(dtype)
    mask = torch.arange(33)[None, :] < torch.tensor([33, 20])[:, None]
    with torch.inference_mode():
        _, plan = mod._attention_plan(x, True, False)
        assert plan.mode == mode and plan.reason == FallbackReason.UNSUPPORTED_DEVICE
        out = mod(x, mask, causal=True)
        ref = baseline_forward(mod, x, mask, True)
    assert torch.equal(out, ref)


def test_parameter_names_match_baseline():
    mod = B200FusedSelfAttention(32, 2)
    assert set(mod.state_dict()) == {f"{p}.{w}" for p in ("q_proj", "k_proj", "v_proj", "out_proj")
                                     for w in ("weight", "bias")}


def test_model_scoped_layer_index_is_checked():
    spec = AttentionModelSpec(1, 32, 32, 2, 32, 1, True)
    mod = B200FusedSelfAttention(32, 2, model_spec=spec, layer_index=1)
    with pytest.raises(ValueError):
        mod._attention_plan(torch.randn(1, 32, 32), True, False)
    with pytest.raises(ValueError):
        B200FusedSelfAttention(33, 2)


def test_functional_op_rejects_cpu_inputs_loudly():
    from b200_attention import b200_fused_attention

    q = torch.randn(1, 2, 8, 64).bfloat16()
    with pytest.raises(ValueError, match="CUDA"):
        b200_fused_attention(q, q, q)
    with pytest.raises(ValueError, match="scale"):
        b200_fused_attention(q, q, q, scale=-1.0)
    with pytest.raises(TypeError):
        b200_fused_attention(q, q.float(), q)
    with pytest.raises(ValueError):
        b200_fused_attention(q, q, q, valid_token_mask=torch.ones(1, 7, dtype=torch.bool))


def test_error_word_survives_inference_mode(monkeypatch):
    """The per-device error word is created as a normal tensor even when the
    first kernel call happens under torch.inference_mode(), so it can be
    cleared outside it (unpinned CPU memory stands in for the pinned word)."""
    from b200_attention import fused_attention as fa

    real_zeros = torch.zeros

    def fake_zeros(*args, **kwargs):
        assert kwargs.pop("pin_memory", False), "the error word lives in pinned host memory"
        return real_zeros(*args, **kwargs)

    monkeypatch.setattr(fa, "_error_words", {})
    monkeypatch.setattr(fa.torch, "zeros", fake_zeros)
    with torch.inference_mode():
        word = fa.device_error_word(torch.device("cuda", 0))
    monkeypatch.undo()
    assert not word.is_inference()
    word.zero_()


def test_operator_is_a_torch_custom_op_with_the_reference_exception_types():
    """The operator is torch.ops.b200.fused_attention (C++ over the C ABI): the
    reference's ValueError / TypeError contract holds through the dispatcher."""
    from b200_attention.fused_attention import _attention_op

    op = _attention_op()
    assert op is torch.ops.b200.fused_attention
    schema = str(op.default._schema)
    assert "Tensor? valid_token_mask" in schema and "int error_word" in schema
    q = torch.randn(1, 2, 8, 64).bfloat16()
    with pytest.raises(ValueError, match="same \\[B, H, S, D\\] shape"):
        op(q, q[:, :1], q, None, False, None, False, False, None, 0)
    with pytest.raises(TypeError, match="same dtype"):
        op(q, q.half(), q, None, False, None, False, False, None, 0)
    with pytest.raises(TypeError, match="floating-point"):
        op(q.int(), q.int(), q.int(), None, False, None, False, False, None, 0)
    with pytest.raises(TypeError, match="torch.bool"):
        op(q, q, q, torch.ones(1, 8), False, None, False, False, None, 0)
    with pytest.raises(ValueError, match="scale must be positive"):
        op(q, q, q, None, False, 0.0, False, False, None, 0)
    with pytest.raises(ValueError, match="CUDA tensors"):
        op(q, q, q, None, False, None, False, False, None, 0)
