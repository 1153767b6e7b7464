"""Pre-LN decoder stack around the attention path (the end-to-end caller).

This is the organiser's benchmark model (torch_transformer_benchmark.py:
BaselineTransformerBlock :126-146, BaselineTransformer :149-171) with its
attention module replaced by ``B200FusedSelfAttention``, the way the harness's
``UserOptimizedTransformer`` seam does (:174-330).  Parameter names match the
organiser's (``layers.{i}.norm1/attention/norm2/ffn_in/ffn_out``,
``final_norm``), so a state dict moves between the two models unchanged.

Per block: ``x + attention(norm1(x))`` then ``x + ffn_out(gelu(ffn_in(norm2(x))))``,
padded rows zeroed after each block and after the final LayerNorm.

With ``fused_epilogues`` (the default) and the attention on its sm_100a path,
a block runs its LayerNorms on the B200 LayerNorm kernel (``b200_layer_norm``)
and the elementwise steps inside the fused linear kernel (``b200_linear``)
where that measured faster than cuBLAS plus the separate passes at the
end-to-end shapes: ``out_proj`` with its residual add (and the padded-row
handling), ``ffn_in`` with the exact GELU, and ``ffn_out`` with its residual
add and padded-row zeroing when a padding mask is given (without a mask,
``ffn_out`` is a plain cuBLAS GEMM followed by the add).  The QKV projection
stays one cuBLAS GEMM.  Every rounding point of the unfused sequence is kept.
An optional
token embedding in front serves the end-to-end configuration (vocabulary 32000,
uniform random token ids); the reference model itself starts from hidden
states, so parity is defined from the hidden states onward.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional, Type

import torch
import torch.nn as nn
import torch.nn.functional as F

from .attention_dispatch import AttentionModelSpec
from .layernorm import b200_layer_norm, layer_norm_supported
from .linear import b200_linear, linear_supported
from .modules import B200FusedSelfAttention


@dataclass(frozen=True)
class DecoderConfig:
    batch_size: int
    seq_len: int
    d_model: int
    num_heads: int
    ffn_dim: int
    num_layers: int
    causal: bool
    vocab_size: Optional[int] = None

    def attention_spec(self) -> AttentionModelSpec:
        return AttentionModelSpec(batch_size=self.batch_size, sequence_length=self.seq_len,
                                  d_model=self.d_model, num_heads=self.num_heads,
                                  ffn_dim=self.ffn_dim, num_layers=self.num_layers,
                                  causal=self.causal)

    def forward_flops(self) -> float:
        """Matmul FLOPs of one forward: QKV and output projections, FFN, and
        attention over visible (query, key) pairs (halved when causal)."""
        tokens = self.batch_size * self.seq_len
        proj = 2.0 * tokens * self.d_model * self.d_model * 4
        ffn = 2.0 * tokens * self.d_model * self.ffn_dim * 2
        attn = 4.0 * self.batch_size * self.seq_len * self.seq_len * self.d_model
        if self.causal:
            attn /= 2
        return self.num_layers * (proj + ffn + attn)


class DecoderBlock(nn.Module):
    def __init__(self, d_model: int, num_heads: int, ffn_dim: int, *,
                 attention_cls: Type[nn.Module] = B200FusedSelfAttention,
                 model_spec: Optional[AttentionModelSpec] = None,
                 layer_index: Optional[int] = None, fused_epilogues: bool = True) -> None:
        super().__init__()
        self.fused_epilogues = fused_epilogues
        self.norm1 = nn.LayerNorm(d_model)
        if model_spec is not None:
            self.attention = attention_cls(d_model, num_heads, model_spec=model_spec,
                                           layer_index=layer_index)
        else:
            self.attention = attention_cls(d_model, num_heads)
        self.norm2 = nn.LayerNorm(d_model)
        self.ffn_in = nn.Linear(d_model, ffn_dim)
        self.ffn_out = nn.Linear(ffn_dim, d_model)

    def forward(self, x: torch.Tensor, valid_token_mask: Optional[torch.Tensor],
                causal: bool) -> torch.Tensor:
        if self._fusable(x):
            h = b200_layer_norm(x, self.norm1.weight, self.norm1.bias, self.norm1.eps)
            fused = self.attention.residual_forward(h, x, valid_token_mask, causal)
            if fused is not None:
                return self._fused_ffn(fused, valid_token_mask)
        x = x + self.attention(self.norm1(x), valid_token_mask, causal)
        x = x + self.ffn_out(F.gelu(self.ffn_in(self.norm2(x)), approximate="none"))
        if valid_token_mask is not None:
            x = x.masked_fill(~valid_token_mask[..., None], 0)
        return x

    def _fusable(self, x: torch.Tensor) -> bool:
        """The block's LayerNorms and linear layers fit the fused kernels for
        input ``x`` (inference on 16-bit CUDA tensors, sizes multiples of 8)."""
        if not self.fused_epilogues or not isinstance(self.attention, B200FusedSelfAttention):
            return False
        if torch.is_grad_enabled() and (x.requires_grad or
                                        any(p.requires_grad for p in self.parameters())):
            return False
        w = self.ffn_out.weight
        return (linear_supported(x, self.ffn_in.weight)
                and layer_norm_supported(x, self.norm1.weight)
                and layer_norm_supported(x, self.norm2.weight)
                and w.device == x.device and w.dtype == x.dtype
                and w.shape[0] % 8 == 0 and w.shape[1] % 8 == 0)

    def _fused_ffn(self, x: torch.Tensor, valid_token_mask: Optional[torch.Tensor]) -> torch.Tensor:
        h = b200_layer_norm(x, self.norm2.weight, self.norm2.bias, self.norm2.eps)
        h = b200_linear(h, self.ffn_in.weight, self.ffn_in.bias, activation="gelu")
        if valid_token_mask is None:
            return x + self.ffn_out(h)
        return b200_linear(h, self.ffn_out.weight, self.ffn_out.bias, residual=x,
                           row_mask=valid_token_mask, masked_rows="zero")


class Decoder(nn.Module):
    """Optional token embedding, ``num_layers`` pre-LN blocks, final LayerNorm."""

    def __init__(self, config: DecoderConfig, *,
                 attention_cls: Type[nn.Module] = B200FusedSelfAttention,
                 model_scoped_plans: bool = True, fused_epilogues: bool = True) -> None:
        super().__init__()
        self.config = config
        spec = config.attention_spec() if model_scoped_plans else None
        self.embed = nn.Embedding(config.vocab_size, config.d_model) if config.vocab_size else None
        self.layers = nn.ModuleList([
            DecoderBlock(config.d_model, config.num_heads, config.ffn_dim,
                         attention_cls=attention_cls, model_spec=spec,
                         layer_index=i if spec is not None else None,
                         fused_epilogues=fused_epilogues)
            for i in range(config.num_layers)])
        self.final_norm = nn.LayerNorm(config.d_model)

    def forward(self, x: torch.Tensor,
                valid_token_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        """``x``: hidden states [B, S, d_model], or token ids [B, S] when the
        model has an embedding."""
        if self.embed is not None and not torch.is_floating_point(x):
            x = self.embed(x)
        fused = len(self.layers) > 0 and self.layers[0]._fusable(x)
        for layer in self.layers:
            x = layer(x, valid_token_mask, self.config.causal)
        if fused and layer_norm_supported(x, self.final_norm.weight):
            x = b200_layer_norm(x, self.final_norm.weight, self.final_norm.bias,
                                self.final_norm.eps)
        else:
            x = self.final_norm(x)
        if valid_token_mask is not None:
            x = x.masked_fill(~valid_token_mask[..., None], 0)
        return x


def init_normal_(model: nn.Module, std: float = 0.02, seed: Optional[int] = None) -> nn.Module:
    """Random-init weights N(0, std), biases zero, LayerNorm weight one (the
    end-to-end configuration's "random-init weights N(0, 0.02)")."""
    gen = None
    if seed is not None:
        gen = torch.Generator(device="cpu").manual_seed(seed)
    with torch.no_grad():
        for mod in model.modules():
            if isinstance(mod, (nn.Linear, nn.Embedding)):
                w = torch.randn(mod.weight.shape, generator=gen) * std
                mod.weight.copy_(w.to(mod.weight.dtype))
                if getattr(mod, "bias", None) is not None:
                    mod.bias.zero_()
            elif isinstance(mod, nn.LayerNorm):
                mod.weight.fill_(1.0)
                mod.bias.zero_()
    return model
