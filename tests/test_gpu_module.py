"""Module adapter on the GPU: SM100_FUSED is planned and runs the native kernel.

Mirrors the reference's fake-fallback detector (test/test_triton_fused_attention.py:124-138):
torch.matmul is patched to raise, so a silent fallback to dense PyTorch fails
the test.  Values are compared with the organiser's operation order.
"""

from unittest import mock

import pytest
import torch
import torch.nn as nn

from b200_attention.attention_dispatch import AttentionMode, AttentionModelSpec
from b200_attention.modules import B200FusedSelfAttention
from oracle.reference_attention import reference_attention
from b200_attention.fused_attention import b200_fused_attention
from parity import assert_close, seeded_qkv

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _baseline(mod, x, mask, causal):
    B, S, d = x.shape
    H = mod.num_heads
    heads = lambda t: t.view(B, S, H, d // H).transpose(1, 2).contiguous().cpu()
    ctx = reference_attention(heads(mod.q_proj(x)), heads(mod.k_proj(x)), heads(mod.v_proj(x)),
                              None if mask is None else mask.cpu(), causal, (d // H) ** -0.5)
    out = mod.out_proj(ctx.to(DEV).transpose(1, 2).contiguous().view(B, S, d))
    if mask is not None:
        out = out.masked_fill(~mask[..., None], 0)
    return out


@pytest.mark.parametrize("d_model,heads", [(1024, 16), (1024, 8)])
def test_module_uses_sm100_kernel(d_model, heads):
    torch.manual_seed(1)
    B, S = 2, 300
    spec = AttentionModelSpec(B, S, d_model, heads, 4 * d_model, 1, True)
    mod = B200FusedSelfAttention(d_model, heads, model_spec=spec, layer_index=0).to(DEV, torch.bfloat16).eval()
    for p in mod.parameters():
        nn.init.normal_(p, std=0.02)
    x = torch.randn(B, S, d_model, device=DEV, dtype=torch.bfloat16)
    mask = torch.arange(S, device=DEV)[None, :] < torch.tensor([300, 170], device=DEV)[:, None]
    with torch.inference_mode():
        _, plan = mod._attention_plan(x, True, False)
        assert plan.mode == AttentionMode.SM100_FUSED
        with mock.patch("torch.matmul", side_effect=AssertionError("dense fallback")):
            out = mod(x, mask, causal=True)
        torch.cuda.synchronize()
        ref = _baseline(mod, x, mask, True)
    assert_close(out, ref, "module")


def test_stacked_blocks_match_baseline_order():
    """Two pre-LN blocks (the organiser's block, torch_transformer_benchmark.py:126-146)."""
    torch.manual_seed(2)
    B, S, d, H = 2, 512, 256, 4
    spec = AttentionModelSpec(B, S, d, H, 4 * d, 2, True)
    layers = []
    for i in range(2):
        blk = nn.ModuleDict(dict(norm1=nn.LayerNorm(d), norm2=nn.LayerNorm(d),
                                 attention=B200FusedSelfAttention(d, H, model_spec=spec, layer_index=i),
                                 ffn_in=nn.Linear(d, 4 * d), ffn_out=nn.Linear(4 * d, d)))
        layers.append(blk.to(DEV, torch.bfloat16).eval())
    x0 = torch.randn(B, S, d, device=DEV, dtype=torch.bfloat16)
    mask = torch.ones(B, S, dtype=torch.bool, device=DEV)

    def run(attn):
        x = x0
        for blk in layers:
            x = x + attn(blk["attention"], blk["norm1"](x))
            x = x + blk["ffn_out"](torch.nn.functional.gelu(blk["ffn_in"](blk["norm2"](x))))
        return x

    with torch.inference_mode():
        fused = run(lambda m, h: m(h, mask, True))
        ref = run(lambda m, h: _baseline(m, h, mask, True))
    diff = (fused.float() - ref.float()).abs()
    assert float(diff.mean()) < 2e-2 and float(diff.max()) < 0.25


@pytest.mark.gpu
def test_operator_replays_in_a_cuda_graph():
    """The operator launches on the caller's stream with no allocation (given
    ``out``) and no host synchronisation, so it can be captured in a CUDA graph;
    replays must equal eager calls bit for bit."""
    dev = torch.device("cuda", 0)
    q, k, v = seeded_qkv((2, 4, 384, 128), torch.bfloat16, 21, device=dev)
    out = torch.empty((2, 384, 4, 128), device=dev, dtype=torch.bfloat16)
    eager = b200_fused_attention(q, k, v, None, True, output_bshd=True).clone()
    graph = torch.cuda.CUDAGraph()
    stream = torch.cuda.Stream(dev)
    stream.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(stream):
        b200_fused_attention(q, k, v, None, True, output_bshd=True, out=out)
        stream.synchronize()
        with torch.cuda.graph(graph, stream=stream):
            b200_fused_attention(q, k, v, None, True, output_bshd=True, out=out)
    torch.cuda.current_stream(dev).wait_stream(stream)
    out.zero_()
    graph.replay()
    torch.cuda.synchronize(dev)
    assert torch.equal(out, eager)
    q.mul_(0.5)  # new inputs in the same buffers: a replay sees them
    graph.replay()
    torch.cuda.synchronize(dev)
    assert torch.equal(out, b200_fused_attention(q, k, v, None, True, output_bshd=True))


@pytest.mark.gpu
@pytest.mark.parametrize("batch,d_model,heads,seq_len", [(64, 128, 4, 128), (64, 128, 16, 128)])
def test_published_matrix_shapes_with_small_heads(batch, d_model, heads, seq_len):
    """The reference's announced benchmark cases mostly use d_model 128 with 4
    heads (D = 32) or 16 heads (D = 8); on a B200 they plan the sm_100a kernel
    (narrow heads read as zero-extended tiles) and must match the baseline order."""
    dev = torch.device("cuda", 0)
    torch.manual_seed(3)
    mod = B200FusedSelfAttention(d_model, heads).to(dev, torch.bfloat16).eval()
    x = torch.randn(batch, seq_len, d_model, device=dev, dtype=torch.bfloat16)
    with torch.inference_mode():
        _, plan = mod._attention_plan(x, True, False)
        assert plan.mode == AttentionMode.SM100_FUSED
        out = mod(x, None, causal=True)
        B, S, d = x.shape
        hd = d // heads
        split = lambda t: t.view(B, S, heads, hd).transpose(1, 2).contiguous()
        ctx = reference_attention(split(mod.q_proj(x)).cpu(), split(mod.k_proj(x)).cpu(),
                                  split(mod.v_proj(x)).cpu(), None, True, hd ** -0.5)
        ref = mod.out_proj(ctx.to(dev).transpose(1, 2).contiguous().view(B, S, d))
    assert_close(out, ref, f"d_model={d_model} heads={heads}")
