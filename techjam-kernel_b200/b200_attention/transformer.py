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
a block runs its LayerNorms on the B200 LayerNorm kernel (``b200_layer_norm``;
without a padding mask the residual add that ends a block runs in the same pass
as the next block's first norm, ``b200_add_layer_norm``) and the elementwise
steps inside the fused linear kernel (``b200_linear``)
where that measured faster than cuBLAS plus the separate passes at the
end-to-end shapes: ``out_proj`` with its residual add (and the padded-row
handling), ``ffn_in`` with the exact GELU, and ``ffn_out`` with its residual
add and padded-row zeroing when a padding mask is given (without a mask,
``ffn_out`` is a plain cuBLAS GEMM whose output is added in that norm pass).
The QKV projection
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
from .layernorm import b200_add_layer_norm, b200_layer_norm, layer_norm_supported
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
            fused = self.fused_body(x, h, valid_token_mask, causal)
            if fused is not None:
                x, pending = fused
                return x if pending is None else x + pending
        x = x + self.attention(self.norm1(x), valid_token_mask, causal)
        x = x + self.ffn_out(F.gelu(self.ffn_in(self.norm2(x)), approximate="none"))
        if valid_token_mask is not None:
            x = x.masked_fill(~valid_token_mask[..., None], 0)
        return x

    def fused_body(self, x: torch.Tensor, h: torch.Tensor,
                   valid_token_mask: Optional[torch.Tensor], causal: bool):
        """The block after its first LayerNorm (``h = norm1(x)``) on the fused
        kernels.  Returns ``(x_next, pending)``: without a padding mask the last
        residual add is left ``pending`` (the ffn_out output, to be added to
        ``x_next`` by the caller, where it can be fused with the next norm);
        with a mask it is done in ffn_out's epilogue and ``pending`` is None.
        Returns None when the attention is not on its sm_100a path."""
        x1 = self.attention.residual_forward(h, x, valid_token_mask, causal)
        if x1 is None:
            return None
        g = b200_layer_norm(x1, self.norm2.weight, self.norm2.bias, self.norm2.eps)
        g = b200_linear(g, self.ffn_in.weight, self.ffn_in.bias, activation="gelu")
        if valid_token_mask is None:
            return x1, self.ffn_out(g)
        return b200_linear(g, self.ffn_out.weight, self.ffn_out.bias, residual=x1,
                           row_mask=valid_token_mask, masked_rows="zero"), None

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
        fused = (len(self.layers) > 0 and all(layer._fusable(x) for layer in self.layers)
                 and layer_norm_supported(x, self.final_norm.weight))
        if fused:
            x = self._forward_fused(x, valid_token_mask)
        else:
            x = self._forward_layers(x, valid_token_mask)
        if valid_token_mask is not None:
            x = x.masked_fill(~valid_token_mask[..., None], 0)
        return x

    def _forward_layers(self, x, valid_token_mask):
        for layer in self.layers:
            x = layer(x, valid_token_mask, self.config.causal)
        return self.final_norm(x)

    def _forward_fused(self, x, valid_token_mask):
        """The blocks on the fused kernels.  Without a padding mask, the
        residual add that ends each block runs in the same pass as the next
        block's first LayerNorm (or the final norm): ``b200_add_layer_norm``
        reads the block's residual stream and its ffn_out output once and
        writes the rounded sum and its normalisation."""
        pending = None  # ffn_out output whose residual add with x is still due
        for layer in self.layers:
            n1 = layer.norm1
            if pending is None:
                h = b200_layer_norm(x, n1.weight, n1.bias, n1.eps)
            else:
                x, h = b200_add_layer_norm(x, pending, n1.weight, n1.bias, n1.eps)
            step = layer.fused_body(x, h, valid_token_mask, self.config.causal)
            if step is None:  # this layer's attention is not on the sm_100a path
                x = layer(x, valid_token_mask, self.config.causal)
                pending = None
            else:
                x, pending = step
        fn = self.final_norm
        if pending is None:
            return b200_layer_norm(x, fn.weight, fn.bias, fn.eps)
        return b200_add_layer_norm(x, pending, fn.weight, fn.bias, fn.eps)[1]


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
