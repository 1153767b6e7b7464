"""CPU oracle for the attention forward — TEST INFRASTRUCTURE ONLY.

This module restates, in the reference's exact operation order, the PyTorch
attention that defines the values the sm_100a kernel must reproduce.  Only
``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may
import it, and only as the checker or the timed CPU baseline; the product path
never calls it.

The value definition is ``_reference_attention`` in the reference
(model/triton_fused_attention.py:1256-1285), identical to the attention core of
the organiser's ``BaselineSelfAttention.forward``
(torch_transformer_benchmark.py:86-113):

    q, k, v made contiguous                         (:1269-1271)
    scores = matmul(q, k^T) * scale                 (:1272)  dtype matmul, then
                                                    the scale multiply in dtype
    scores.masked_fill(triu(ones(S,S), 1), -inf)    (:1273-1279) when causal
    scores.masked_fill(~mask[:,None,None,:], -inf)  (:1280-1283) when masked
    probs = softmax(scores.float(), -1).to(dtype)   (:1284)
    out = matmul(probs, v)                          (:1285)

The arithmetic is torch's CPU kernels (matmul, masked_fill, softmax).  The
reference pins no torch version (no requirements or lock file); it is anchored
here by golden vectors produced by importing the reference itself
(tests/golden/make_golden.py) and checked bit-for-bit in tests.
"""

from __future__ import annotations

from typing import Optional

import torch


def reference_attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    valid_token_mask: Optional[torch.Tensor],
    causal: bool,
    scale: float,
) -> torch.Tensor:
    """Dense oracle; follows model/triton_fused_attention.py:1256-1285 step by step."""
    q_ref = q.contiguous()
    k_ref = k.contiguous()
    v_ref = v.contiguous()
    scores = torch.matmul(q_ref, k_ref.transpose(-2, -1))
    probabilities = reference_softmax(scores, valid_token_mask, scale, causal)
    return torch.matmul(probabilities, v_ref)


def reference_softmax(
    scores: torch.Tensor,
    valid_token_mask: Optional[torch.Tensor],
    scale: float,
    causal: bool,
) -> torch.Tensor:
    """The softmax stage of the value definition on unscaled scores ``[B, H, S, S]``
    (model/triton_fused_attention.py:1272-1284; torch_transformer_benchmark.py:98-112):
    the scale multiply in the scores' dtype, causal triu(1) and key-mask
    positions set to -inf, fp32 softmax, rounded back to the dtype.  This is
    also what the reference's row-softmax seam computes
    (model/triton_softmax.py:19-96, 99-161), which takes the unscaled scores."""
    seq_len = scores.shape[-1]
    scores = scores * scale
    if causal:
        causal_mask = torch.ones((seq_len, seq_len), device=scores.device,
                                 dtype=torch.bool).triu(diagonal=1)
        scores = scores.masked_fill(causal_mask, float("-inf"))
    if valid_token_mask is not None:
        scores = scores.masked_fill(~valid_token_mask[:, None, None, :], float("-inf"))
    return torch.softmax(scores.float(), dim=-1).to(scores.dtype)


def reference_softmax_rows(
    scores_rows: torch.Tensor,
    valid_token_mask: Optional[torch.Tensor],
    scale: float,
    causal: bool,
    row_start: int,
) -> torch.Tensor:
    """``reference_softmax`` for the query rows ``[row_start, row_start + R)``
    only (``scores_rows`` is ``[B, H, R, S]``), each element computed exactly as
    in the dense form; the bounded form for long rows."""
    rows, seq_len = scores_rows.shape[-2], scores_rows.shape[-1]
    scores = scores_rows * scale
    if causal:
        r = torch.arange(row_start, row_start + rows, device=scores.device)[:, None]
        c = torch.arange(seq_len, device=scores.device)[None, :]
        scores = scores.masked_fill(c > r, float("-inf"))
    if valid_token_mask is not None:
        scores = scores.masked_fill(~valid_token_mask[:, None, None, :], float("-inf"))
    return torch.softmax(scores.float(), dim=-1).to(scores.dtype)


def reference_attention_rows(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    valid_token_mask: Optional[torch.Tensor],
    causal: bool,
    scale: float,
    row_start: int,
    row_end: int,
) -> torch.Tensor:
    """Oracle for query rows [row_start, row_end) only, same operation order.

    Bounded-memory form for long sequences (the reference's own bounded oracle
    is _blocked_fp32_attention_rows, model/triton_fused_attention.py:1456-1504):
    the score block is [B, H, rows, S] instead of [B, H, S, S].  Each element of
    the block is computed exactly as in ``reference_attention``.
    """
    q_rows = q[:, :, row_start:row_end].contiguous()
    k_ref = k.contiguous()
    v_ref = v.contiguous()
    seq_len = k.shape[2]
    scores = torch.matmul(q_rows, k_ref.transpose(-2, -1)) * scale
    if causal:
        rows = torch.arange(row_start, row_end, device=q.device)[:, None]
        cols = torch.arange(seq_len, device=q.device)[None, :]
        scores = scores.masked_fill(cols > rows, float("-inf"))
    if valid_token_mask is not None:
        scores = scores.masked_fill(~valid_token_mask[:, None, None, :], float("-inf"))
    probabilities = torch.softmax(scores.float(), dim=-1).to(q.dtype)
    return torch.matmul(probabilities, v_ref)


def reference_attention_blocked(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    valid_token_mask: Optional[torch.Tensor],
    causal: bool,
    scale: float,
    rows_per_block: int = 256,
) -> torch.Tensor:
    """Full output assembled from ``reference_attention_rows`` blocks."""
    seq_len = q.shape[2]
    out = torch.empty_like(q, memory_format=torch.contiguous_format)
    for start in range(0, seq_len, rows_per_block):
        end = min(seq_len, start + rows_per_block)
        out[:, :, start:end] = reference_attention_rows(q, k, v, valid_token_mask, causal, scale, start, end)
    return out


def zero_masked_rows(out: torch.Tensor, valid_token_mask: Optional[torch.Tensor]) -> torch.Tensor:
    """Rows whose own mask bit is False set to 0 ([B,H,S,D] layout): the value the
    reference's module leaves there after out_proj (model/triton_fused_attention.py:2460-2461)."""
    if valid_token_mask is None:
        return out
    return out.masked_fill(~valid_token_mask[:, None, :, None], 0)


def attention_flops(batch: int, heads: int, seq_len: int, head_dim: int, causal: bool,
                    valid_lengths: Optional[list[int]] = None) -> float:
    """Algorithmic FLOPs: 4*B*H*S^2*D (QK^T and PV), halved for causal; with
    prefix key masks and skipped padded queries, 4*H*D*sum(L_b^2)."""
    if valid_lengths is not None:
        return 4.0 * heads * head_dim * float(sum(int(L) * int(L) for L in valid_lengths))
    flops = 4.0 * batch * heads * seq_len * seq_len * head_dim
    return flops / 2.0 if causal else flops
