"""Module adapter: a drop-in for the reference's ``TritonFusedSelfAttention``.

Same constructor ``(d_model, num_heads, *, model_spec=None, layer_index=None)``
(model/triton_fused_attention.py:2169-2206), same learned parameter names
(``q_proj``, ``k_proj``, ``v_proj``, ``out_proj``) for strict state-dict copies,
same ``forward(x, valid_token_mask=None, causal=False)`` and the same per-call
plan cache keyed by dtype, device, shape, causality and autograd (:2216-2285).

Per layer the planner picks the executor:

* ``SM100_FUSED``: one GEMM computes Q, K and V together against the three
  projection weights stacked ([3d, d], cached until a weight changes); q/k/v
  are strided head views of its [B, S, 3, H, D] output (no copies; the
  reference keeps per-projection views, :2287-2292); the sm_100a kernel writes
  the context directly in the [B, S, H, D] layout ``out_proj`` consumes;
  padded query rows are zeroed after ``out_proj`` exactly as the reference
  does (:2456-2461).  ``residual_forward`` additionally folds the block's
  residual add into the output projection (one fused linear kernel).
* ``EXACT_REFERENCE`` / ``FP32_BASELINE_EXACT``: the planner routes inputs the
  kernel does not cover (autograd, fp32, other head sizes, non-CUDA devices) to
  the organiser's PyTorch operation order, as the reference planner does.
* the reference's Triton/Gluon modes (capability >= 12): not shipped here;
  raises ``NotImplementedError``.
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn

from .attention_dispatch import (AttentionMode, AttentionModelSpec, AttentionRuntime, PlanScope,
                                 select_attention_stack_plan)
from .fused_attention import b200_fused_attention
from .linear import b200_linear, linear_supported

_DTYPE_NAMES = {torch.float16: "float16", torch.bfloat16: "bfloat16", torch.float32: "float32"}


def _dtype_name(dtype: torch.dtype) -> str:
    return _DTYPE_NAMES.get(dtype, str(dtype).removeprefix("torch."))


def _exact_attention_core(q, k, v, valid_token_mask, causal: bool, scale: float):
    """The organiser's attention order (torch_transformer_benchmark.py:96-113) on
    contiguous [B,H,S,D] heads; executed only for planner-selected exact modes."""
    seq_len = q.shape[2]
    scores = torch.matmul(q, k.transpose(-2, -1)) * scale
    if causal:
        upper = torch.ones((seq_len, seq_len), device=q.device, dtype=torch.bool).triu(diagonal=1)
        scores = scores.masked_fill(upper, float("-inf"))
    if valid_token_mask is not None:
        scores = scores.masked_fill(~valid_token_mask[:, None, None, :], float("-inf"))
    probs = torch.softmax(scores.float(), dim=-1).to(q.dtype)
    return torch.matmul(probs, v)


class B200FusedSelfAttention(nn.Module):
    """Baseline-compatible self-attention whose core runs on the sm_100a kernel."""

    def __init__(self, d_model: int, num_heads: int, *,
                 model_spec: Optional[AttentionModelSpec] = None,
                 layer_index: Optional[int] = None) -> None:
        super().__init__()
        if d_model % num_heads != 0:
            raise ValueError("d_model must be divisible by num_heads")
        self.d_model = d_model
        self.num_heads = num_heads
        self.head_dim = d_model // num_heads
        self.scale = self.head_dim ** -0.5
        self._attention_model_spec = model_spec
        self._attention_layer_index = layer_index
        self._plan_key: Optional[tuple] = None
        self._plan_value: Optional[tuple] = None
        self._qkv_key: Optional[tuple] = None
        self._qkv_value: Optional[tuple] = None
        self.q_proj = nn.Linear(d_model, d_model, bias=True)
        self.k_proj = nn.Linear(d_model, d_model, bias=True)
        self.v_proj = nn.Linear(d_model, d_model, bias=True)
        self.out_proj = nn.Linear(d_model, d_model, bias=True)

    # ------------------------------------------------------------ planning
    def _attention_plan(self, x: torch.Tensor, causal: bool, needs_autograd: bool):
        batch, seq_len, d_model = x.shape
        device_index = x.device.index if x.device.type == "cuda" else None
        key = (x.dtype, x.device.type, device_index, batch, seq_len, d_model, causal, needs_autograd)
        if self._plan_key == key:
            return self._plan_value
        spec = self._attention_model_spec
        if spec is None:
            spec = AttentionModelSpec(batch_size=batch, sequence_length=seq_len, d_model=self.d_model,
                                      num_heads=self.num_heads, ffn_dim=self.d_model, num_layers=1,
                                      causal=causal)
            scope, layer = PlanScope.STANDALONE, 0
        else:
            scope, layer = PlanScope.MODEL, self._attention_layer_index
            if layer is None:
                raise ValueError("model-scoped attention requires a layer index")
        capability = None
        if x.device.type == "cuda" and torch.cuda.is_available():
            capability = torch.cuda.get_device_capability(x.device)
        runtime = AttentionRuntime(batch_size=batch, sequence_length=seq_len, d_model=d_model,
                                   dtype=_dtype_name(x.dtype), device_type=x.device.type,
                                   device_capability=capability, needs_autograd=needs_autograd,
                                   causal=causal)
        stack = select_attention_stack_plan(spec, runtime, scope)
        if layer < 0 or layer >= len(stack.layers):
            raise ValueError(f"attention layer index {layer} is outside the selected plan")
        self._plan_key, self._plan_value = key, (stack, stack.layers[layer])
        return self._plan_value

    # ------------------------------------------------------------- forward
    def _stacked_qkv(self):
        """[3d, d] weight and [3d] bias of the q, k, v projections, rebuilt
        only when one of them changed (identity, storage or version)."""
        params = (self.q_proj.weight, self.k_proj.weight, self.v_proj.weight,
                  self.q_proj.bias, self.k_proj.bias, self.v_proj.bias)
        key = tuple((id(t), t.data_ptr(), t._version, t.dtype, t.device) for t in params)
        if self._qkv_key != key:
            with torch.no_grad():
                weight = torch.cat(params[:3], dim=0)
                bias = torch.cat(params[3:], dim=0)
            self._qkv_key, self._qkv_value = key, (weight, bias)
        return self._qkv_value

    def _heads_view(self, projected: torch.Tensor) -> torch.Tensor:
        batch, seq_len, _ = projected.shape
        return projected.view(batch, seq_len, self.num_heads, self.head_dim).transpose(1, 2)

    def _sm100_context(self, x: torch.Tensor, valid_token_mask: Optional[torch.Tensor],
                       causal: bool) -> torch.Tensor:
        """Attention context [B, S, d] before ``out_proj`` on the sm_100a path."""
        batch, seq_len, _ = x.shape
        weight, bias = self._stacked_qkv()
        qkv = torch.nn.functional.linear(x, weight, bias).view(
            batch, seq_len, 3, self.num_heads, self.head_dim)
        q, k, v = (qkv[:, :, t].transpose(1, 2) for t in range(3))
        context = b200_fused_attention(q, k, v, valid_token_mask, causal, self.scale,
                                       output_bshd=True)
        return context.view(batch, seq_len, self.d_model)

    def _plan_mode(self, x: torch.Tensor, causal: bool) -> AttentionMode:
        needs_autograd = torch.is_grad_enabled() and (
            x.requires_grad or any(p.requires_grad for p in self.parameters()))
        _, plan = self._attention_plan(x, causal, needs_autograd)
        return plan.mode

    def residual_forward(self, x: torch.Tensor, residual: torch.Tensor,
                         valid_token_mask: Optional[torch.Tensor] = None,
                         causal: bool = False) -> Optional[torch.Tensor]:
        """``residual + self(x, valid_token_mask, causal)``, the first half of
        the reference block (torch_transformer_benchmark.py:141), with the
        output projection, its bias, the padded-row zeroing and the residual add
        in one fused linear kernel (rows whose mask is False keep ``residual``
        unchanged, as ``residual + 0`` does).  Returns None when this call does
        not take the sm_100a path; the caller then runs the unfused sequence."""
        if self._plan_mode(x, causal) != AttentionMode.SM100_FUSED:
            return None
        if not linear_supported(x, self.out_proj.weight) or residual.shape != x.shape \
                or residual.dtype != x.dtype:
            return None
        context = self._sm100_context(x, valid_token_mask, causal)
        return b200_linear(context, self.out_proj.weight, self.out_proj.bias, residual=residual,
                           row_mask=valid_token_mask, masked_rows="residual")

    def forward(self, x: torch.Tensor, valid_token_mask: Optional[torch.Tensor] = None,
                causal: bool = False) -> torch.Tensor:
        batch, seq_len, _ = x.shape
        mode = self._plan_mode(x, causal)

        if mode == AttentionMode.SM100_FUSED:
            context = self._sm100_context(x, valid_token_mask, causal)
        elif mode in (AttentionMode.EXACT_REFERENCE, AttentionMode.FP32_BASELINE_EXACT):
            q = self._heads_view(self.q_proj(x)).contiguous()
            k = self._heads_view(self.k_proj(x)).contiguous()
            v = self._heads_view(self.v_proj(x)).contiguous()
            context = _exact_attention_core(q, k, v, valid_token_mask, causal, self.scale)
            context = context.transpose(1, 2).contiguous().view(batch, seq_len, self.d_model)
        else:
            raise NotImplementedError(
                f"attention mode {mode} runs on the reference's Triton/Gluon (sm_120) stack, "
                "which this package does not ship")
        output = self.out_proj(context)
        if valid_token_mask is not None:
            output = output.masked_fill(~valid_token_mask[..., None], 0)
        return output
