"""Planner boundary: same API and plans as the reference planner, plus SM100_FUSED.

Golden plans come from the reference planner itself (tests/golden/planner_plans.json,
made by tests/golden/make_golden.py) for its 14 published shapes x dtype x
capability x scope.  For capability 12.0 and 9.0 our planner must return the
same plans; for 10.0 (B200) the reference returns exact/cuda_capability and our
planner selects SM100_FUSED wherever the sm_100a kernel's envelope holds.
"""

import json
from pathlib import Path

import pytest

from b200_attention.attention_dispatch import (AttentionFamily,
                                               AttentionMode, AttentionModelSpec, AttentionRuntime,
                                               FallbackReason, PlanScope, clear_plan_cache,
                                               select_attention_stack_plan, sm100_supports)

PLANS = json.loads((Path(__file__).resolve().parent / "golden" / "planner_plans.json").read_text())


def _plan_dict(sp):
    return {"execution": sp.execution,
            "layers": [{"mode": p.mode.value, "family": p.family.value,
                        "reason": p.reason.value if p.reason else None,
                        "explanation": p.explanation,
                        "launch": None if p.launch is None else {
                            f: getattr(p.launch, f) for f in ("block_m", "block_n", "num_warps",
                                                              "num_stages", "query_block_size",
                                                              "output_layout")}}
                       for p in sp.layers]}


def _select(entry):
    spec = AttentionModelSpec(*entry["spec"])
    rt = AttentionRuntime(spec.batch_size, spec.sequence_length, spec.d_model, entry["dtype"],
                          "cuda", tuple(entry["capability"]), False, spec.causal)
    return spec, select_attention_stack_plan(spec, rt, entry["scope"])


@pytest.mark.parametrize("entry", [e for e in PLANS if e["capability"][0] != 10],
                         ids=lambda e: f"case{e['case']}-{e['dtype']}-cc{e['capability'][0]}-{e['scope']}")
def test_reference_plans_reproduced(entry):
    _, sp = _select(entry)
    assert _plan_dict(sp) == {"execution": entry["execution"], "layers": entry["layers"]}


@pytest.mark.parametrize("entry", [e for e in PLANS if e["capability"][0] == 10],
                         ids=lambda e: f"case{e['case']}-{e['dtype']}-{e['scope']}")
def test_b200_plans(entry):
    spec, sp = _select(entry)
    in_envelope = sm100_supports(entry["dtype"], spec.head_dim)
    # the reference runs every B200 shape on its exact PyTorch path
    assert {l["reason"] for l in entry["layers"]} == {"cuda_capability"}
    if in_envelope:
        assert {p.mode for p in sp.layers} == {AttentionMode.SM100_FUSED}
        assert {p.family for p in sp.layers} == {AttentionFamily.SM100_TILED}
        assert all(p.reason is None and p.launch.block_m == 128 for p in sp.layers)
        assert sp.execution == "batched"
    else:
        assert {p.family for p in sp.layers} == {AttentionFamily.EXACT}
        assert all(p.reason in (FallbackReason.UNSUPPORTED_DTYPE, FallbackReason.UNVALIDATED_SHAPE)
                   for p in sp.layers)


def _rt(dtype="bfloat16", cap=(10, 0), device="cuda", autograd=False, B=8, S=2048, d=2048, causal=True):
    return AttentionRuntime(B, S, d, dtype, device, cap, autograd, causal)


def test_b200_gates():
    spec = AttentionModelSpec(8, 2048, 2048, 16, 8192, 2, True)  # D = 128
    assert select_attention_stack_plan(spec, _rt()).layers[0].mode == AttentionMode.SM100_FUSED
    assert select_attention_stack_plan(spec, _rt("float16")).layers[0].mode == AttentionMode.SM100_FUSED
    fp32 = select_attention_stack_plan(spec, _rt("float32")).layers[0]
    # fp32 runs the TF32 instance for head dims up to 64 only
    assert (fp32.mode, fp32.reason) == (AttentionMode.FP32_BASELINE_EXACT, FallbackReason.UNVALIDATED_SHAPE)
    d64 = AttentionModelSpec(8, 2048, 1024, 16, 4096, 2, True)  # D = 64
    fp32_64 = select_attention_stack_plan(d64, _rt("float32", d=1024)).layers[0]
    assert fp32_64.mode == AttentionMode.SM100_FUSED and fp32_64.launch.num_stages == 5
    assert select_attention_stack_plan(d64, _rt("float64", d=1024)).layers[0].reason == \
        FallbackReason.UNSUPPORTED_DTYPE
    ag = select_attention_stack_plan(spec, _rt(autograd=True)).layers[0]
    assert (ag.mode, ag.reason) == (AttentionMode.EXACT_REFERENCE, FallbackReason.AUTOGRAD)
    mism = select_attention_stack_plan(spec, _rt(S=1024)).layers[0]
    assert mism.reason == FallbackReason.SHAPE_MISMATCH
    cpu = select_attention_stack_plan(spec, _rt(device="cpu", cap=None)).layers[0]
    assert cpu.reason == FallbackReason.UNSUPPORTED_DEVICE
    d32 = AttentionModelSpec(8, 2048, 512, 16, 512, 1, True)  # D = 32: the 64-wide instance
    assert select_attention_stack_plan(d32, _rt(d=512)).layers[0].mode == AttentionMode.SM100_FUSED
    d12 = AttentionModelSpec(8, 2048, 192, 16, 512, 1, True)  # 12: not a multiple of 8
    assert select_attention_stack_plan(d12, _rt(d=192)).layers[0].reason == FallbackReason.UNVALIDATED_SHAPE
    d256 = AttentionModelSpec(8, 2048, 4096, 16, 512, 1, True)
    assert select_attention_stack_plan(d256, _rt(d=4096)).layers[0].reason == FallbackReason.UNVALIDATED_SHAPE
    noncausal = AttentionModelSpec(16, 4096, 4096, 32, 4096, 1, False)
    plan = select_attention_stack_plan(noncausal, _rt(B=16, S=4096, d=4096, causal=False))
    assert plan.layers[0].mode == AttentionMode.SM100_FUSED


def test_e2e_config_plans_every_layer_on_sm100():
    # 12 layers, d_model 1024, 16 heads (D = 64), FFN 4096
    spec = AttentionModelSpec(8, 2048, 1024, 16, 4096, 12, True)
    plan = select_attention_stack_plan(spec, _rt(d=1024))
    assert len(plan.layers) == 12 and {p.mode for p in plan.layers} == {AttentionMode.SM100_FUSED}
    launch = plan.layers[0].launch
    assert (launch.block_m, launch.block_n, launch.num_warps, launch.num_stages) == (128, 128, 11, 10)


def test_cache_and_invalid_specs():
    clear_plan_cache()
    spec = AttentionModelSpec(1, 128, 128, 4, 128, 4, True)
    rt = AttentionRuntime(1, 128, 128, "float32", "cuda", (12, 0), False, True)
    a = select_attention_stack_plan(spec, rt, scope=PlanScope.STANDALONE)
    assert a is select_attention_stack_plan(spec, rt, scope="standalone")
    with pytest.raises(ValueError):
        AttentionModelSpec(1, 32, 33, 2, 32, 1, True)
    with pytest.raises(ValueError):
        AttentionModelSpec(1, 32, 32, 2, 32, 0, True)
    with pytest.raises(ValueError):
        AttentionRuntime(0, 32, 32, "float32", "cuda", (12, 0), False, True)
    assert str(AttentionMode.SM100_FUSED) == "sm100_fused"
