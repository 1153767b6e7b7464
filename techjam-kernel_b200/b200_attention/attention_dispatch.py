"""Attention planner: which executor each layer runs (torch-free, pure, cached).

This keeps the public API of the reference planner
(model/attention_dispatch.py): the value types ``AttentionModelSpec``,
``AttentionRuntime``, ``KernelLaunch``, ``AttentionPlan``,
``AttentionStackPlan``, the enums ``PlanScope``, ``AttentionFamily``,
``AttentionMode``, ``FallbackReason``, and the entry point
``select_attention_stack_plan(spec, runtime, scope)`` (:563-575) with its
``lru_cache`` (:513) and ``clear_plan_cache`` (:578).

Added for B200: one mode, ``SM100_FUSED`` (family ``SM100_TILED``), chosen for
every layer when the runtime is a CUDA device of compute capability 10.x and
the dtype/head dimension lie inside the sm_100a kernel's envelope.  On other
capabilities the reference's published policy is reproduced unchanged: its
runtime gates (:357-386), its 17 published per-layer rules (:254-273), its
generic envelope (:399-459) and its family/reason attachment (:471-510).  The
modes that policy names for capability >= 12 are executed by the reference's
Triton stack, which this package does not ship; the module adapter refuses
them explicitly.
"""

from __future__ import annotations

from dataclasses import dataclass
from enum import Enum
from functools import lru_cache
from typing import Optional


class _TextEnum(str, Enum):
    def __str__(self) -> str:
        return self.value


class PlanScope(_TextEnum):
    MODEL = "model"
    STANDALONE = "standalone"


class AttentionFamily(_TextEnum):
    EXACT = "exact"
    SHORT_FULL_ROW = "short_full_row"
    SHORT_SMALL_HEAD = "short_small_head"
    LONG_TILED = "long_tiled"
    D256_SPECIALIZED = "d256_specialized"
    SM100_TILED = "sm100_tiled"


class AttentionMode(_TextEnum):
    EXACT_REFERENCE = "exact_reference"
    FP32_BASELINE_EXACT = "fp32_baseline_exact"
    FP16_BLOCKED_EXACT = "fp16_blocked_exact"
    BF16_BLOCKED_EXACT = "bf16_blocked_exact"
    FP16_FULL_ROW = "fp16_full_row"
    BF16_FULL_ROW = "bf16_full_row"
    FP32_FULL_ROW_TF32 = "fp32_full_row_tf32"
    FP32_SMALL_HEAD_TF32 = "fp32_small_head_tf32"
    FP16_TWO_PASS = "fp16_two_pass"
    FP16_LONG_TILED = "fp16_long_tiled"
    BF16_LONG_TILED = "bf16_long_tiled"
    FP32_LONG_TILED = "fp32_long_tiled"
    SM100_FUSED = "sm100_fused"


class FallbackReason(_TextEnum):
    UNSUPPORTED_DTYPE = "unsupported_dtype"
    UNSUPPORTED_DEVICE = "unsupported_device"
    CUDA_CAPABILITY = "cuda_capability"
    AUTOGRAD = "autograd"
    SHAPE_MISMATCH = "shape_mismatch"
    UNVALIDATED_SHAPE = "unvalidated_shape"
    FP32_D128_REJECTED = "fp32_d128_rejected"
    FP32_D256_REJECTED = "fp32_d256_rejected"
    BF16_D32_LONG_UNVALIDATED = "bf16_d32_long_unvalidated"
    RESIDUAL_STACK_POLICY = "residual_stack_policy"


# Envelope of the sm_100a kernel; the C ABI's b200_attn_query answers the same
# question and a CPU test keeps the two in agreement.
SM100_DTYPES = ("bfloat16", "float16", "float32")
# 16-bit: every multiple of 8 up to 128 (narrower heads run the 64- or
# 128-wide kernel instance with the missing columns read as zeros by TMA);
# fp32 (TF32 products): every multiple of 8 up to 64.
SM100_HEAD_DIMS = tuple(range(8, 129, 8))
SM100_FP32_HEAD_DIMS = tuple(range(8, 65, 8))


def sm100_supports(dtype: str, head_dim: int) -> bool:
    """Whether the sm_100a kernel computes attention for (dtype, head_dim)."""
    if dtype == "float32":
        return head_dim in SM100_FP32_HEAD_DIMS
    return dtype in SM100_DTYPES and head_dim in SM100_HEAD_DIMS
SM100_CAPABILITY_MAJOR = 10
# Launch shape of the sm_100a kernel (the C ABI's b200_attn_launch_shape
# reports the same values; a CPU test keeps the two in agreement): 128-row
# query tiles, two per CTA, 128-key K/V tiles, 11 warps (two softmax
# warpgroups, a TMA warp and two tcgen05 issuer warps), and a ring of K/V
# slots (one K or one V tile each) whose depth depends on the instance.
SM100_BLOCK_M = 128
SM100_BLOCK_N = 128
SM100_NUM_WARPS = 11


def sm100_ring_slots(head_dim: int, dtype: str = "bfloat16") -> int:
    """K/V ring slots of the kernel instance that serves (dtype, head_dim):
    the 16-bit 64-wide instance (head dims up to 64) holds 10, the 128-wide
    one and the fp32 instance (32 KB tiles) 5."""
    if dtype == "float32":
        return 5
    return 10 if head_dim <= 64 else 5


@dataclass(frozen=True, slots=True)
class AttentionModelSpec:
    """Configured Transformer shape (reference :65-109)."""

    batch_size: int
    sequence_length: int
    d_model: int
    num_heads: int
    ffn_dim: int
    num_layers: int
    causal: bool

    def __post_init__(self) -> None:
        dims = (self.batch_size, self.sequence_length, self.d_model, self.num_heads,
                self.ffn_dim, self.num_layers)
        if min(dims) <= 0:
            raise ValueError("model dimensions and layer count must be positive")
        if self.d_model % self.num_heads:
            raise ValueError("d_model must be divisible by num_heads")

    @property
    def head_dim(self) -> int:
        if self.num_heads <= 0 or self.d_model % self.num_heads:
            return 0
        return self.d_model // self.num_heads

    def key(self) -> tuple[object, ...]:
        return (self.batch_size, self.sequence_length, self.d_model, self.num_heads,
                self.ffn_dim, self.num_layers, self.causal)


@dataclass(frozen=True, slots=True)
class AttentionRuntime:
    """Runtime facts that can make a configured plan ineligible (reference :112-146)."""

    batch_size: int
    sequence_length: int
    d_model: int
    dtype: str
    device_type: str
    device_capability: Optional[tuple[int, int]]
    needs_autograd: bool
    causal: bool
    bf16_fused_min_length: int = 100000

    def __post_init__(self) -> None:
        if min(self.batch_size, self.sequence_length, self.d_model) <= 0:
            raise ValueError("runtime dimensions must be positive")
        if self.bf16_fused_min_length <= 0:
            raise ValueError("bf16_fused_min_length must be positive")

    def key(self) -> tuple[object, ...]:
        return (self.batch_size, self.sequence_length, self.d_model, self.dtype,
                self.device_type, self.device_capability, self.needs_autograd, self.causal,
                self.bf16_fused_min_length)


@dataclass(frozen=True, slots=True)
class KernelLaunch:
    """Launch values carried by a plan (reference :149-158)."""

    block_m: Optional[int] = None
    block_n: Optional[int] = None
    num_warps: Optional[int] = None
    num_stages: Optional[int] = None
    query_block_size: Optional[int] = None
    output_layout: str = "bshd"


@dataclass(frozen=True, slots=True)
class AttentionPlan:
    """One layer's family and mode (reference :161-176)."""

    layer_index: int
    family: AttentionFamily
    mode: AttentionMode
    launch: Optional[KernelLaunch] = None
    reason: Optional[FallbackReason] = None
    explanation: Optional[str] = None

    @property
    def label(self) -> str:
        return self.mode.value


@dataclass(frozen=True, slots=True)
class AttentionStackPlan:
    """Per-layer plans plus the whole-stack execution policy (reference :179-187)."""

    layers: tuple[AttentionPlan, ...]
    execution: str = "batched"

    @property
    def microbatch_size(self) -> Optional[int]:
        return 1 if self.execution == "microbatch_one" else None


# ----------------------------------------------------------------------------
# Published per-shape policy of the reference (model/attention_dispatch.py:254-273).
# Data, kept identical: (dtype, batch sizes, S, d_model, heads, ffn, layers, modes).
_M = AttentionMode
_PUBLISHED_RULES: tuple[tuple, ...] = (
    ("float16", (1, 4, 16, 64, 128, 10000), 128, 128, 4, 128, 4, (_M.FP16_FULL_ROW,) * 4),
    ("bfloat16", (1, 4, 16, 64, 128, 10000), 128, 128, 4, 128, 4, (_M.BF16_FULL_ROW,) * 4),
    ("float32", (1, 4, 16, 64, 128), 128, 128, 4, 128, 4,
     (_M.FP32_BASELINE_EXACT,) + (_M.FP32_FULL_ROW_TF32,) * 3),
    ("float32", (10000,), 128, 128, 4, 128, 4,
     (_M.FP32_BASELINE_EXACT,) * 2 + (_M.FP32_FULL_ROW_TF32,) * 2),
    ("float32", (64,), 128, 32, 4, 32, 4,
     (_M.FP32_BASELINE_EXACT,) + (_M.FP32_SMALL_HEAD_TF32,) * 3),
    ("float32", (64,), 128, 1024, 4, 1024, 4, (_M.FP32_BASELINE_EXACT,) * 4),
    ("float32", (64,), 128, 128, 1, 128, 4, (_M.FP32_BASELINE_EXACT,) * 4),
    ("float32", (64,), 128, 128, 2, 128, 4, (_M.FP32_FULL_ROW_TF32,) * 4),
    ("float32", (64,), 128, 128, 16, 128, 4, (_M.FP32_SMALL_HEAD_TF32,) * 4),
    ("float32", (64,), 32, 128, 4, 128, 4,
     (_M.FP32_BASELINE_EXACT,) + (_M.FP32_FULL_ROW_TF32,) * 3),
    ("float32", (64,), 1024, 128, 4, 128, 4, (_M.FP32_LONG_TILED,) * 4),
    ("float16", (64,), 1024, 128, 4, 128, 4,
     (_M.FP16_BLOCKED_EXACT,) + (_M.FP16_TWO_PASS,) * 3),
    ("float16", (32,), 100000, 1024, 16, 1024, 2, (_M.FP16_LONG_TILED,) * 2),
    ("bfloat16", (32,), 100000, 1024, 16, 1024, 2, (_M.BF16_LONG_TILED,) * 2),
    ("float32", (32,), 100000, 1024, 16, 1024, 2, (_M.FP32_LONG_TILED,) * 2),
    ("float32", (1,), 1024, 1024, 16, 1024, 2, (_M.FP32_LONG_TILED,) * 2),
    ("float32", (1,), 100000, 1024, 16, 1024, 2, (_M.FP32_LONG_TILED,) * 2),
)

# The one published shape the reference runs as whole-stack batch-of-one
# (reference :283-286 of its runtime gate and :540-550).
_MICROBATCH_SHAPE = (32, 100000, 1024, 16, 1024, 2)

_FAMILY = {
    _M.FP16_FULL_ROW: AttentionFamily.SHORT_FULL_ROW,
    _M.BF16_FULL_ROW: AttentionFamily.SHORT_FULL_ROW,
    _M.FP32_FULL_ROW_TF32: AttentionFamily.SHORT_FULL_ROW,
    _M.FP32_SMALL_HEAD_TF32: AttentionFamily.SHORT_SMALL_HEAD,
    _M.FP16_TWO_PASS: AttentionFamily.LONG_TILED,
    _M.FP16_LONG_TILED: AttentionFamily.LONG_TILED,
    _M.BF16_LONG_TILED: AttentionFamily.LONG_TILED,
    _M.FP32_LONG_TILED: AttentionFamily.LONG_TILED,
    _M.BF16_BLOCKED_EXACT: AttentionFamily.EXACT,
    _M.FP16_BLOCKED_EXACT: AttentionFamily.EXACT,
    _M.EXACT_REFERENCE: AttentionFamily.EXACT,
    _M.FP32_BASELINE_EXACT: AttentionFamily.EXACT,
    _M.SM100_FUSED: AttentionFamily.SM100_TILED,
}

_REASON_TEXT = {
    FallbackReason.UNSUPPORTED_DTYPE: "dtype is outside the validated attention modes",
    FallbackReason.UNSUPPORTED_DEVICE: "validated kernels require CUDA",
    FallbackReason.CUDA_CAPABILITY: "validated Gluon/Triton kernels require CUDA capability >= sm120",
    FallbackReason.AUTOGRAD: "inference-only kernels are disabled when autograd is required",
    FallbackReason.SHAPE_MISMATCH: "runtime shape or causal mode does not match the configured plan",
}


def _rule_matches(rule: tuple, spec: AttentionModelSpec, dtype: str) -> bool:
    r_dtype, batches, seq, d_model, heads, ffn, layers, _ = rule
    return (r_dtype == dtype and spec.batch_size in batches and spec.causal
            and (spec.sequence_length, spec.d_model, spec.num_heads, spec.ffn_dim,
                 spec.num_layers) == (seq, d_model, heads, ffn, layers))


def _sm100_launch(head_dim: int, dtype: str = "bfloat16") -> KernelLaunch:
    # num_stages = K/V ring slots (one K or one V tile per slot)
    return KernelLaunch(block_m=SM100_BLOCK_M, block_n=SM100_BLOCK_N, num_warps=SM100_NUM_WARPS,
                        num_stages=sm100_ring_slots(head_dim, dtype), output_layout="bshd")


def _published_launch(mode: AttentionMode, spec: AttentionModelSpec,
                      dtype: str = "bfloat16") -> Optional[KernelLaunch]:
    """Launch metadata the reference attaches per mode (reference :303-354)."""
    S, D = spec.sequence_length, spec.head_dim
    if mode in (_M.FP16_FULL_ROW, _M.BF16_FULL_ROW):
        return KernelLaunch(block_m=32 if S <= 32 else 64, block_n=1 << (S - 1).bit_length(), num_warps=4)
    if mode == _M.FP32_FULL_ROW_TF32:
        if S == 32 and D == 32:
            block_m, warps = 32, 8
        elif S <= 32:
            block_m, warps = 16, 4
        elif S <= 64:
            block_m, warps = (16 if D <= 32 else 32), 4
        else:
            block_m, warps = (32 if D <= 32 else 64), 4
        return KernelLaunch(block_m=block_m, block_n=1 << (S - 1).bit_length(), num_warps=warps)
    if mode == _M.FP32_SMALL_HEAD_TF32:
        return {4: KernelLaunch(block_m=64, block_n=64, num_warps=2),
                16: KernelLaunch(block_m=64, block_n=128, num_warps=4)}.get(
            spec.num_heads, KernelLaunch(block_m=32, block_n=128, num_warps=4))
    if mode in (_M.FP16_TWO_PASS, _M.FP16_LONG_TILED):
        return KernelLaunch(block_m=64, block_n=64, num_warps=4, num_stages=3)
    if mode == _M.BF16_LONG_TILED:
        return KernelLaunch(block_m=32, block_n=32, num_warps=4, num_stages=1)
    if mode == _M.FP32_LONG_TILED:
        return KernelLaunch(block_m=64, block_n=32, num_warps=4, num_stages=3 if D == 32 else 2)
    if mode in (_M.FP16_BLOCKED_EXACT, _M.BF16_BLOCKED_EXACT):
        return KernelLaunch(query_block_size=16, output_layout="bhsd")
    if mode == _M.SM100_FUSED:
        return _sm100_launch(D, dtype)
    return None


def _shape_reason(spec: AttentionModelSpec, rt: AttentionRuntime) -> Optional[FallbackReason]:
    # A batch-of-one call inside the published whole-stack microbatch is valid.
    microbatch_sample = (
        (spec.batch_size, spec.sequence_length, spec.d_model, spec.num_heads, spec.ffn_dim,
         spec.num_layers) == _MICROBATCH_SHAPE and spec.causal and rt.batch_size == 1
    )
    if (not (rt.batch_size == spec.batch_size or microbatch_sample)
            or rt.sequence_length != spec.sequence_length or rt.d_model != spec.d_model
            or rt.causal != spec.causal):
        return FallbackReason.SHAPE_MISMATCH
    return None


def _runtime_reason(spec: AttentionModelSpec, rt: AttentionRuntime) -> Optional[FallbackReason]:
    """Gates of the reference planner (reference :357-386), in its order."""
    if rt.dtype not in ("float16", "bfloat16", "float32"):
        return FallbackReason.UNSUPPORTED_DTYPE
    if rt.device_type != "cuda":
        return FallbackReason.UNSUPPORTED_DEVICE
    if rt.device_capability is None or rt.device_capability[0] < 12:
        return FallbackReason.CUDA_CAPABILITY
    if rt.needs_autograd:
        return FallbackReason.AUTOGRAD
    return _shape_reason(spec, rt)


def _sm100_reason(spec: AttentionModelSpec, rt: AttentionRuntime) -> Optional[FallbackReason]:
    """Gates for the sm_100a kernel; None means every layer runs SM100_FUSED."""
    if rt.dtype not in ("float16", "bfloat16", "float32"):
        return FallbackReason.UNSUPPORTED_DTYPE
    if rt.needs_autograd:
        return FallbackReason.AUTOGRAD
    shape = _shape_reason(spec, rt)
    if shape is not None:
        return shape
    if rt.dtype not in SM100_DTYPES:
        return FallbackReason.UNSUPPORTED_DTYPE
    if not sm100_supports(rt.dtype, spec.head_dim):
        return FallbackReason.UNVALIDATED_SHAPE
    return None


def _is_sm100(rt: AttentionRuntime) -> bool:
    return (rt.device_type == "cuda" and rt.device_capability is not None
            and rt.device_capability[0] == SM100_CAPABILITY_MAJOR)


def _generic_mode(spec: AttentionModelSpec, rt: AttentionRuntime, scope: PlanScope
                  ) -> tuple[Optional[AttentionMode], Optional[FallbackReason], str]:
    """Shape envelope outside the published rules (reference :399-459)."""
    dtype, S, D = rt.dtype, spec.sequence_length, spec.head_dim
    if S >= 257:
        if not spec.causal:
            return None, FallbackReason.UNVALIDATED_SHAPE, \
                "long-sequence kernels are validated only for causal attention"
        if dtype == "float16" and D == 32 and S == 1024:
            return _M.FP16_TWO_PASS, None, "validated D=32 long attention keeps the two-pass reduction"
        if dtype == "float16" and D == 64:
            return _M.FP16_LONG_TILED, None, "validated FP16 bounded long-sequence kernel"
        if dtype == "bfloat16" and D == 64:
            if S >= rt.bf16_fused_min_length:
                return _M.BF16_LONG_TILED, None, "validated BF16 bounded long-sequence kernel"
            return _M.BF16_BLOCKED_EXACT, None, \
                "BF16 bounded exact reduction preserves baseline rounding below the fused threshold"
        if dtype == "bfloat16" and D == 32:
            return None, FallbackReason.BF16_D32_LONG_UNVALIDATED, "no validated BF16 D=32 long-sequence kernel"
        return None, FallbackReason.UNVALIDATED_SHAPE, \
            "no validated long-sequence kernel for this dtype/head dimension"
    if S in (32, 64, 128):
        if dtype in ("float16", "bfloat16") and D in (16, 32, 64, 128):
            mode = _M.FP16_FULL_ROW if dtype == "float16" else _M.BF16_FULL_ROW
            return mode, None, "validated short full-row Gluon kernel"
        if dtype == "float32" and S == 128 and D == 8:
            return _M.FP32_SMALL_HEAD_TF32, None, "validated padded D=8 TF32 small-head kernel"
        if dtype == "float32" and D in (16, 32, 64, 128):
            standalone_ok = {(32, 32), (128, 32), (32, 64), (64, 64), (128, 64), (128, 8)}
            if scope == PlanScope.STANDALONE and (S, D) in standalone_ok:
                return _M.FP32_FULL_ROW_TF32, None, "standalone validated FP32 full-row kernel"
            return None, FallbackReason.UNVALIDATED_SHAPE, "FP32 model shape has no published residual-stack policy"
    if dtype == "float32" and D == 256:
        return None, FallbackReason.FP32_D256_REJECTED, \
            "experimental FP32 D=256 kernel is not correctness/performance certified"
    return None, FallbackReason.UNVALIDATED_SHAPE, "shape is outside the validated attention envelope"


def _exact(index: int, dtype: str, reason: FallbackReason, explanation: str) -> AttentionPlan:
    mode = _M.FP32_BASELINE_EXACT if dtype == "float32" else _M.EXACT_REFERENCE
    return AttentionPlan(index, AttentionFamily.EXACT, mode, None, reason, explanation)


def _plan(index: int, mode: AttentionMode, spec: AttentionModelSpec,
          explanation: Optional[str] = None, dtype: str = "bfloat16") -> AttentionPlan:
    """Attach family, launch and residual-stack reasons (reference :471-510)."""
    reason = None
    if mode == _M.FP32_BASELINE_EXACT and spec.d_model == 1024 and spec.num_heads == 4:
        reason = FallbackReason.FP32_D256_REJECTED
        explanation = "FP32 D=256 chunked candidate is not correctness/performance certified"
    elif mode == _M.FP32_BASELINE_EXACT and spec.num_heads == 1:
        reason = FallbackReason.FP32_D128_REJECTED
        explanation = "FP32 D=128 Gluon candidate regressed the protected benchmark"
    elif mode in (_M.FP32_BASELINE_EXACT, _M.FP16_BLOCKED_EXACT):
        reason = FallbackReason.RESIDUAL_STACK_POLICY
    return AttentionPlan(index, _FAMILY[mode], mode, _published_launch(mode, spec, dtype), reason,
                         explanation)


@lru_cache(maxsize=256)
def _select_cached(spec: AttentionModelSpec, rt: AttentionRuntime, scope: PlanScope) -> AttentionStackPlan:
    layers = range(spec.num_layers)

    if _is_sm100(rt):
        reason = _sm100_reason(spec, rt)
        if reason is None:
            text = "sm_100a tcgen05/TMEM fused attention kernel"
            return AttentionStackPlan(tuple(_plan(i, _M.SM100_FUSED, spec, text, rt.dtype)
                                            for i in layers))
        text = _REASON_TEXT.get(reason, "outside the sm_100a kernel envelope")
        return AttentionStackPlan(tuple(_exact(i, rt.dtype, reason, text) for i in layers))

    reason = _runtime_reason(spec, rt)
    if reason is not None:
        text = _REASON_TEXT.get(reason, reason.value)
        return AttentionStackPlan(tuple(_exact(i, rt.dtype, reason, text) for i in layers))

    if scope != PlanScope.STANDALONE:
        for rule in _PUBLISHED_RULES:
            if _rule_matches(rule, spec, rt.dtype):
                plans = []
                for i, mode in enumerate(rule[7]):
                    text = None
                    if mode == _M.FP32_BASELINE_EXACT:
                        text = "published residual-stack policy keeps this layer in organizer operation order"
                    elif mode == _M.FP16_BLOCKED_EXACT:
                        text = "first D=32 long layer keeps the exact FP16 score/probability boundary"
                    plans.append(_plan(i, mode, spec, text))
                shape = (spec.batch_size, spec.sequence_length, spec.d_model, spec.num_heads,
                         spec.ffn_dim, spec.num_layers)
                execution = ("microbatch_one" if shape == _MICROBATCH_SHAPE and rt.batch_size == 32
                             else "batched")
                return AttentionStackPlan(tuple(plans), execution)

    mode, reason, text = _generic_mode(spec, rt, scope)
    if mode is not None:
        return AttentionStackPlan(tuple(_plan(i, mode, spec, text) for i in layers))
    return AttentionStackPlan(tuple(
        _exact(i, rt.dtype, reason or FallbackReason.UNVALIDATED_SHAPE, text) for i in layers))


def select_attention_stack_plan(
    spec: AttentionModelSpec,
    runtime: AttentionRuntime,
    scope: PlanScope = PlanScope.MODEL,
) -> AttentionStackPlan:
    """Plan every layer's attention mode and the stack's execution policy.

    Pure and cached by (spec, runtime, scope); the only production policy
    authority.  Invalid specs raise ``ValueError`` at construction.
    """
    return _select_cached(spec, runtime, PlanScope(scope))


def clear_plan_cache() -> None:
    """Drop cached plans (tests that inspect cache behaviour)."""
    _select_cached.cache_clear()
