"""The decoder block with its linear layers on the fused kernel (out_proj +
residual, ffn_in + GELU, ffn_out + residual + padded-row zeroing) against the
same weights with cuBLAS linear layers and separate elementwise passes.

Both runs keep every rounding point of the unfused sequence; they differ by
the GEMMs' fp32 summation order, the LayerNorm's two-pass statistics and the
GELU's erfc formula, each a last-bit effect that the following layers carry
on.  Bounds: mean-abs <= 2e-3 (the repository's parity bound) and max-abs <=
2^-6 of the largest output magnitude (two bf16 units in the last place of the
largest value); padded rows must be exactly zero after every block.
"""

import pytest
import torch

from b200_attention import linear as linear_mod
from b200_attention.transformer import Decoder, DecoderConfig, init_normal_
from parity import MEAN_ABS, compare

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
CFG = DecoderConfig(2, 512, 1024, 16, 4096, 2, True)


def _pair(cfg):
    fused = init_normal_(Decoder(cfg), seed=7).to(device=DEV, dtype=torch.bfloat16).eval()
    plain = Decoder(cfg, fused_epilogues=False).to(device=DEV, dtype=torch.bfloat16).eval()
    plain.load_state_dict(fused.state_dict())
    return fused, plain


@pytest.mark.parametrize("padded", [False, True])
def test_fused_blocks_match_unfused(padded, monkeypatch):
    fused, plain = _pair(CFG)
    gen = torch.Generator().manual_seed(11)
    x = torch.randn(CFG.batch_size, CFG.seq_len, CFG.d_model, generator=gen).to(DEV, torch.bfloat16)
    mask = None
    if padded:
        lengths = torch.tensor([CFG.seq_len, CFG.seq_len // 3])
        mask = (torch.arange(CFG.seq_len)[None, :] < lengths[:, None]).to(DEV)
        x = x.masked_fill(~mask[..., None], 0)
    calls = []
    real = linear_mod.b200_linear

    def counting(*args, **kwargs):
        calls.append(kwargs.get("activation"))
        return real(*args, **kwargs)

    monkeypatch.setattr("b200_attention.transformer.b200_linear", counting)
    monkeypatch.setattr("b200_attention.modules.b200_linear", counting)
    with torch.inference_mode():
        out = fused(x, mask)
        ref = plain(x, mask)
    torch.cuda.synchronize()
    # per block: out_proj (+residual), ffn_in (+GELU), and ffn_out when masked
    assert len(calls) == CFG.num_layers * (3 if padded else 2)
    stats = compare(out, ref)
    assert stats["mean_abs"] <= MEAN_ABS, stats
    assert stats["max_abs"] <= 2.0**-6 * ref.float().abs().max().item(), stats
    if mask is not None:
        assert torch.equal(out[~mask], torch.zeros_like(out[~mask]))


def test_autograd_takes_the_unfused_path():
    fused, plain = _pair(DecoderConfig(1, 256, 1024, 16, 4096, 1, True))
    x = torch.randn(1, 256, 1024, device=DEV, dtype=torch.bfloat16, requires_grad=True)
    out = fused(x)
    out.float().sum().backward()
    assert x.grad is not None and torch.isfinite(x.grad.float()).all()


@pytest.mark.parametrize("padded", [False, True])
def test_fused_path_never_falls_back_to_torch_norm_or_gelu(padded, monkeypatch):
    """The reference's fake-fallback detector (test/test_triton_fused_attention.py:124-138):
    with torch's LayerNorm and GELU made to raise, the fused decoder must still
    run, so none of its norms or activations silently took the torch path."""
    import torch.nn.functional as F

    fused, _ = _pair(CFG)
    x = torch.randn(CFG.batch_size, CFG.seq_len, CFG.d_model, device=DEV, dtype=torch.bfloat16)
    mask = None
    if padded:
        mask = (torch.arange(CFG.seq_len)[None, :] < torch.tensor([CFG.seq_len, 100])[:, None]).to(DEV)

    def forbidden(*args, **kwargs):
        raise AssertionError("torch fallback used on the fused path")

    monkeypatch.setattr(F, "layer_norm", forbidden)
    monkeypatch.setattr(F, "gelu", forbidden)
    with torch.inference_mode():
        out = fused(x, mask)
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()
