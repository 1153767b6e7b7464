"""Decoder stack around the attention path, on CPU (exact planner modes).

On a CPU device every layer plans the organiser's exact operation order, so
the decoder built on ``B200FusedSelfAttention`` must equal, bit for bit, the
organiser's baseline model (torch_transformer_benchmark.py:126-171) restated
with the oracle's attention (``tests/e2e_models.py``).
"""

import pytest
import torch

from b200_attention.transformer import Decoder, DecoderConfig, init_normal_
from e2e_models import OracleSelfAttention

ORGANISER_KEYS = {
    "layers.0.norm1.weight", "layers.0.norm1.bias",
    "layers.0.attention.q_proj.weight", "layers.0.attention.q_proj.bias",
    "layers.0.attention.k_proj.weight", "layers.0.attention.k_proj.bias",
    "layers.0.attention.v_proj.weight", "layers.0.attention.v_proj.bias",
    "layers.0.attention.out_proj.weight", "layers.0.attention.out_proj.bias",
    "layers.0.norm2.weight", "layers.0.norm2.bias",
    "layers.0.ffn_in.weight", "layers.0.ffn_in.bias",
    "layers.0.ffn_out.weight", "layers.0.ffn_out.bias",
    "final_norm.weight", "final_norm.bias",
}


def _pair(cfg, dtype):
    ours = init_normal_(Decoder(cfg), seed=3).to(dtype).eval()
    base = Decoder(cfg, attention_cls=OracleSelfAttention, model_scoped_plans=False).to(dtype).eval()
    base.load_state_dict(ours.state_dict(), strict=True)
    return ours, base


def test_parameter_names_match_the_organiser_model():
    cfg = DecoderConfig(1, 8, 32, 2, 64, 1, True)
    assert set(Decoder(cfg).state_dict()) == ORGANISER_KEYS


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("causal,lengths", [(True, None), (False, [48, 17])])
def test_cpu_decoder_equals_baseline(dtype, causal, lengths):
    cfg = DecoderConfig(2, 48, 64, 4, 128, 2, causal)
    ours, base = _pair(cfg, dtype)
    gen = torch.Generator().manual_seed(11)
    x = torch.randn(2, 48, 64, generator=gen).to(dtype)
    mask = None
    if lengths:
        mask = torch.arange(48)[None, :] < torch.tensor(lengths)[:, None]
        x = x.masked_fill(~mask[..., None], 0)
    with torch.inference_mode():
        a, b = ours(x, mask), base(x, mask)
    assert torch.equal(a, b)


def test_token_embedding_front():
    cfg = DecoderConfig(2, 16, 32, 2, 64, 1, True, vocab_size=100)
    ours = init_normal_(Decoder(cfg), seed=5).eval()
    tokens = torch.randint(0, 100, (2, 16), generator=torch.Generator().manual_seed(1))
    with torch.inference_mode():
        out = ours(tokens)
        ref = ours(ours.embed(tokens))
    assert out.shape == (2, 16, 32) and torch.equal(out, ref)


def test_forward_flops_of_the_end_to_end_config():
    cfg = DecoderConfig(8, 2048, 1024, 16, 4096, 12, True, vocab_size=32000)
    assert abs(cfg.forward_flops() / 1e12 - 5.772) < 1e-3
