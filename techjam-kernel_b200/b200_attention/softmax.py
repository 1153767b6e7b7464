"""Row softmax over materialised attention scores on the B200
(``include/b200_softmax.h``): the reference's unfused attention seam.

``b200_attention_softmax(scores, valid_token_mask, scale, causal)`` keeps the
signature, checks and exception types of the reference's
``triton_attention_softmax`` (model/triton_softmax.py:99-161): ``scores`` is a
contiguous ``[B, H, S, S]`` CUDA tensor of unscaled ``q k^T`` (fp32, fp16 or
bf16), the scale multiply is rounded to its dtype, causal and key-padding
positions become -inf, and the softmax runs in fp32 with one rounding to the
dtype.  ``B200SoftmaxSelfAttention`` is the reference's ``TritonSelfAttention``
(:164-219) over this kernel: the same constructor, learned parameter names and
forward.  Both are also exported under the reference's names so its seam
(torch_transformer_benchmark.py:185) imports them unchanged.  There is no
fallback: inputs the kernel does not take raise.
"""

from __future__ import annotations

import ctypes
import struct
from typing import Optional

import torch
import torch.nn as nn

from . import _native
from .fused_attention import SUPPORTED_DTYPES, raise_for_code

# b200_softmax_params packed in one call (layout checked against the ctypes
# mirror at import): scores probs, B H S, mask and its two strides, scale,
# dtype, causal, reserved.
_SOFTMAX_LAYOUT = struct.Struct("=2Q3qQ2qfiii")
assert _SOFTMAX_LAYOUT.size == ctypes.sizeof(_native.SoftmaxParams)


def b200_attention_softmax(
    scores: torch.Tensor,
    valid_token_mask: Optional[torch.Tensor],
    scale: float,
    causal: bool,
    *,
    out: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """Scaled, masked, fp32 row softmax of ``scores`` on the B200; a new tensor
    like ``scores`` (or ``out``, which may be ``scores`` itself)."""
    if scores.ndim != 4:
        raise ValueError(f"scores must have shape [B, H, S, S], got {scores.shape}")
    batch, num_heads, query_len, key_len = scores.shape
    if query_len != key_len:
        raise ValueError("self-attention scores must be square in the last two dims")
    if scores.device.type != "cuda":
        raise ValueError("b200_attention_softmax requires CUDA scores")
    if scores.dtype not in SUPPORTED_DTYPES:
        raise TypeError(f"unsupported scores dtype: {scores.dtype}")
    if not scores.is_contiguous():
        raise ValueError("scores must be contiguous")
    if valid_token_mask is not None:
        if valid_token_mask.shape != (batch, key_len):
            raise ValueError(
                "valid_token_mask must have shape "
                f"{(batch, key_len)}, got {tuple(valid_token_mask.shape)}"
            )
        if valid_token_mask.dtype != torch.bool:
            raise TypeError("valid_token_mask must have dtype torch.bool")
        if valid_token_mask.device != scores.device:
            raise ValueError("valid_token_mask and scores must be on the same device")
        if not valid_token_mask.is_contiguous():
            raise ValueError("valid_token_mask must be contiguous")
    if key_len > _native.SOFTMAX_MAX_SEQ:
        raise ValueError(f"sequence length {key_len} is too large for this row kernel")
    if not scale > 0:
        raise ValueError("scale must be positive")
    if out is None:
        out = torch.empty_like(scores)
    elif out.shape != scores.shape or out.dtype != scores.dtype or not out.is_contiguous() \
            or out.device != scores.device:
        raise ValueError("out must be a contiguous tensor like scores")
    if scores.numel() == 0:
        return out
    if valid_token_mask is not None:
        mask, ms0, ms1 = valid_token_mask.data_ptr(), valid_token_mask.stride(0), \
            valid_token_mask.stride(1)
    else:
        mask = ms0 = ms1 = 0
    p = _native.SoftmaxParams()
    _SOFTMAX_LAYOUT.pack_into(p, 0, scores.data_ptr(), out.data_ptr(), batch, num_heads, key_len,
                              mask, ms0, ms1, float(scale), SUPPORTED_DTYPES[scores.dtype],
                              1 if causal else 0, 0)
    lib = _native.load_library()
    rc = lib.b200_softmax_fwd(ctypes.byref(p),
                              ctypes.c_void_p(torch.cuda.current_stream(scores.device).cuda_stream))
    if rc != _native.OK:
        raise_for_code("b200_softmax_fwd", rc, scores.device)
    return out


class B200SoftmaxSelfAttention(nn.Module):
    """Baseline-compatible attention whose softmax stage runs on the B200 row
    kernel: QK^T and PV are torch matmuls over contiguous heads, as in the
    reference's TritonSelfAttention (model/triton_softmax.py:164-219)."""

    def __init__(self, d_model: int, num_heads: int) -> None:
        super().__init__()
        if d_model % num_heads != 0:
            raise ValueError("d_model must be divisible by num_heads")
        self.d_model = d_model
        self.num_heads = num_heads
        self.head_dim = d_model // num_heads
        self.scale = self.head_dim ** -0.5
        self.q_proj = nn.Linear(d_model, d_model, bias=True)
        self.k_proj = nn.Linear(d_model, d_model, bias=True)
        self.v_proj = nn.Linear(d_model, d_model, bias=True)
        self.out_proj = nn.Linear(d_model, d_model, bias=True)

    def _split_heads(self, x: torch.Tensor) -> torch.Tensor:
        batch, seq_len, _ = x.shape
        return x.view(batch, seq_len, self.num_heads, self.head_dim).transpose(1, 2).contiguous()

    def forward(self, x: torch.Tensor, valid_token_mask: Optional[torch.Tensor] = None,
                causal: bool = False) -> torch.Tensor:
        batch, seq_len, _ = x.shape
        q = self._split_heads(self.q_proj(x))
        k = self._split_heads(self.k_proj(x))
        v = self._split_heads(self.v_proj(x))
        scores = torch.matmul(q, k.transpose(-2, -1))
        probabilities = b200_attention_softmax(scores, valid_token_mask, self.scale, causal,
                                               out=scores)
        context = torch.matmul(probabilities, v)
        context = context.transpose(1, 2).contiguous().view(batch, seq_len, self.d_model)
        output = self.out_proj(context)
        if valid_token_mask is not None:
            output = output.masked_fill(~valid_token_mask[..., None], 0)
        return output


# the reference's names (model/triton_softmax.py; seam torch_transformer_benchmark.py:185)
triton_attention_softmax = b200_attention_softmax
TritonSelfAttention = B200SoftmaxSelfAttention
