"""GPU parity of the row-softmax kernel (the reference's unfused attention
seam, model/triton_softmax.py) against the CPU oracle's softmax stage, which
is the value definition's (pinned bit for bit to the reference's outputs through
``oracle.reference_attention``).

Tolerance: both sides compute the softmax in fp32 and round once.  They differ
in the exponential (CUDA's expf is within 2 units in the last place, the CPU's
exp within 1), the division's rounding and the order of the fp32 sum over the
row (relative difference about sqrt(S) * 2^-24, 5e-6 at S = 8192).  A 16-bit
output therefore lies within one unit in the last place of the oracle's value;
an fp32 output within 2e-5 of it, relative.  NaN patterns (rows whose keys are
all masked) must be equal.
"""

import pytest
import torch

from b200_attention import (B200SoftmaxSelfAttention, b200_attention_softmax, read_device_errors)
from oracle.reference_attention import reference_attention, reference_softmax, reference_softmax_rows
from parity import assert_close, prefix_mask, seeded_qkv, unit_in_last_place

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


FP32_RTOL = 2e-5


def assert_within_units(out, ref, units, label):
    """16-bit: within ``units`` units in the last place of ``ref``; fp32:
    within FP32_RTOL of it, relative."""
    o, r = out.float().cpu(), ref.float().cpu()
    assert torch.equal(torch.isnan(o), torch.isnan(r)), f"{label}: NaN pattern differs"
    fin = ~torch.isnan(r)
    d = (o - r).abs()[fin]
    if ref.dtype == torch.float32:
        bound = FP32_RTOL * r[fin].abs()
    else:
        bound = units * unit_in_last_place(r[fin], ref.dtype)
    bound = torch.maximum(bound, torch.full_like(bound, torch.finfo(ref.dtype).tiny))
    assert bool((d <= bound).all()), f"{label}: worst {float((d - bound).max()):.3e}"


def _scores(shape, dtype, seed):
    q, k, _ = seeded_qkv(shape, dtype, seed)
    return torch.matmul(q, k.transpose(-1, -2))  # unscaled, in dtype (CPU)


UNITS = {torch.bfloat16: 1, torch.float16: 1, torch.float32: None}


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("S", [1, 33, 64, 256, 257, 1000, 1024, 2048, 4097, 8192])
@pytest.mark.parametrize("causal,masked", [(True, False), (False, True), (True, True)])
def test_softmax_matches_oracle(dtype, S, causal, masked):
    B, H, D = (2, 2, 64) if S <= 4096 else (2, 1, 64)
    scores = _scores((B, H, S, D), dtype, 100 + S)
    mask = prefix_mask(B, S, [S, max(1, S // 3)]) if masked else None
    ref = reference_softmax(scores, mask, D ** -0.5, causal)
    out = b200_attention_softmax(scores.to(DEV), None if mask is None else mask.to(DEV),
                                 D ** -0.5, causal)
    torch.cuda.synchronize()
    assert out.dtype == dtype and out.shape == scores.shape
    assert_within_units(out, ref, UNITS[dtype], f"{dtype} S={S}")


def test_softmax_in_place_and_fully_masked_rows():
    B, H, S, D = 2, 3, 300, 64
    scores = _scores((B, H, S, D), torch.bfloat16, 7)
    mask = prefix_mask(B, S, [300, 0])  # batch 1: no valid key -> NaN rows
    ref = reference_softmax(scores, mask, 0.125, False)
    sd = scores.to(DEV)
    out = b200_attention_softmax(sd, mask.to(DEV), 0.125, False, out=sd)
    torch.cuda.synchronize()
    assert out is sd and torch.isnan(out[1].float()).all()
    assert_within_units(out, ref, 1, "in place")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_softmax_causal_rows_with_no_visible_key_are_nan(dtype):
    # Causal rows skip the column chunks past their query index; a row whose
    # visible keys are all masked must still be NaN in those chunks too.
    B, H, S, D = 2, 2, 1024, 64
    scores = _scores((B, H, S, D), dtype, 11)
    mask = prefix_mask(B, S, [S, 0])
    ref = reference_softmax(scores, mask, D ** -0.5, True)
    out = b200_attention_softmax(scores.to(DEV), mask.to(DEV), D ** -0.5, True)
    torch.cuda.synchronize()
    assert torch.isnan(out[1].float()).all()
    assert_within_units(out, ref, UNITS[dtype], f"{dtype} causal, no visible key")


@pytest.mark.parametrize("S", [16384, 32768])
def test_softmax_long_rows_in_registers(S):
    scores = _scores((1, 1, S, 32), torch.bfloat16, 11)
    out = b200_attention_softmax(scores.to(DEV), None, 32 ** -0.5, True).cpu()
    for r0 in (0, S // 2, S - 64):
        ref = reference_softmax_rows(scores[:, :, r0:r0 + 64], None, 32 ** -0.5, True, r0)
        assert_within_units(out[:, :, r0:r0 + 64], ref, 1, f"S={S} rows {r0}")


def test_softmax_rows_beyond_the_register_form():
    """S in (32768, 65536]: the three-pass form, fp16 and a key mask."""
    S = 33000
    gen = torch.Generator().manual_seed(13)
    scores = (4 * torch.randn((1, 1, S, S), generator=gen)).half()
    mask = prefix_mask(1, S, [32001])
    out = b200_attention_softmax(scores.to(DEV), mask.to(DEV), 0.5, True).cpu()
    for r0 in (0, 16000, S - 64):
        ref = reference_softmax_rows(scores[:, :, r0:r0 + 64], mask, 0.5, True, r0)
        assert_within_units(out[:, :, r0:r0 + 64], ref, 1, f"long rows {r0}")


def test_seam_attention_matches_reference_attention():
    """matmul -> this softmax -> matmul, the reference's materialised path
    (test/test_triton_fused_attention.py:41-56), against the value definition."""
    q, k, v = seeded_qkv((2, 4, 384, 64), torch.float16, 5)
    mask = prefix_mask(2, 384, [384, 100])
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    probs = b200_attention_softmax(torch.matmul(qd, kd.transpose(-1, -2)), mask.to(DEV), 0.125, True)
    out = torch.matmul(probs, vd)
    torch.cuda.synchronize()
    assert_close(out, reference_attention(q, k, v, mask, True, 0.125), "seam")


def test_module_loads_baseline_weights_and_zeroes_padded_queries():
    """The reference's module test (test/test_triton_fused_attention.py:1120-1150):
    baseline weights load strictly, fp16, padded queries exactly zero."""
    from e2e_models import OracleSelfAttention

    torch.manual_seed(9012)
    base = OracleSelfAttention(128, 2)
    mod = B200SoftmaxSelfAttention(128, 2)
    mod.load_state_dict(base.state_dict(), strict=True)
    base = base.to(DEV).half().eval()
    mod = mod.to(DEV).half().eval()
    x = torch.randn((2, 33, 128), device=DEV, dtype=torch.float16)
    mask = torch.arange(33, device=DEV)[None, :] < torch.tensor([33, 17], device=DEV)[:, None]
    with torch.inference_mode():
        expected = base(x, mask, causal=False)
        actual = mod(x, mask, causal=False)
    torch.cuda.synchronize()
    d = (actual.float() - expected.float()).abs()
    assert bool(((d <= 2e-3) | (d <= 2e-2 * expected.float().abs())).all())
    assert bool((actual[1, 17:] == 0).all())
    assert read_device_errors(DEV) == 0
