"""Baseline attention module for the end-to-end (model-level) parity tests.

``OracleSelfAttention`` is the organiser's ``BaselineSelfAttention``
(torch_transformer_benchmark.py:60-123) with its attention core taken from the
oracle (the reference's operation order).  Plugged into
``b200_attention.transformer.Decoder`` it gives the organiser's baseline model
(torch_transformer_benchmark.py:126-171) with the same parameter names, so one
state dict serves both models.  Test infrastructure only.
"""

from __future__ import annotations

import torch
import torch.nn as nn

from oracle.reference_attention import reference_attention


class OracleSelfAttention(nn.Module):
    def __init__(self, d_model: int, num_heads: int, **_: object) -> None:
        super().__init__()
        self.d_model = d_model
        self.num_heads = num_heads
        self.head_dim = d_model // num_heads
        self.q_proj = nn.Linear(d_model, d_model, bias=True)
        self.k_proj = nn.Linear(d_model, d_model, bias=True)
        self.v_proj = nn.Linear(d_model, d_model, bias=True)
        self.out_proj = nn.Linear(d_model, d_model, bias=True)

    def _heads(self, t: torch.Tensor) -> torch.Tensor:
        b, s, _ = t.shape
        return t.view(b, s, self.num_heads, self.head_dim).transpose(1, 2).contiguous()

    def forward(self, x, valid_token_mask=None, causal=False):
        b, s, _ = x.shape
        ctx = reference_attention(self._heads(self.q_proj(x)), self._heads(self.k_proj(x)),
                                  self._heads(self.v_proj(x)), valid_token_mask, causal,
                                  self.head_dim ** -0.5)
        out = self.out_proj(ctx.transpose(1, 2).contiguous().view(b, s, self.d_model))
        if valid_token_mask is not None:
            out = out.masked_fill(~valid_token_mask[..., None], 0)
        return out
