"""The CPU oracle reproduces the reference's own outputs (golden vectors).

The fixtures were produced by importing the reference and calling its public
operator on CPU (tests/golden/make_golden.py); the oracle must match them
bit for bit.  This pins the oracle before it is trusted as the GPU checker.
"""

import json
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle.reference_attention import (attention_flops, reference_attention,
                                        reference_attention_blocked, reference_attention_rows,
                                        zero_masked_rows)
from tests_golden_io import load_case_inputs

GOLDEN = Path(__file__).resolve().parent / "golden"
META = json.loads((GOLDEN / "attention_cases.json").read_text())
ARRAYS = np.load(GOLDEN / "attention_cases.npz")


def _golden_tensor(case):
    arr = ARRAYS[case["name"]]
    if case["dtype"] == "float32":
        return torch.from_numpy(arr)
    dt = torch.bfloat16 if case["dtype"] == "bfloat16" else torch.float16
    return torch.from_numpy(arr).view(dt)


@pytest.mark.parametrize("case", META["cases"], ids=[c["name"] for c in META["cases"]])
def test_oracle_matches_reference_golden(case):
    q, k, v, mask = load_case_inputs(case)
    D = case["shape"][-1]
    out = reference_attention(q, k, v, mask, case["causal"], D ** -0.5)
    if case["keep_heads"]:
        out = out[:, :case["keep_heads"]]
    gold = _golden_tensor(case)
    assert out.dtype == gold.dtype and out.shape == gold.shape
    # bit-exact, NaN positions included
    assert torch.equal(out.view(torch.int16) if out.dtype != torch.float32 else out.view(torch.int32),
                       gold.view(torch.int16) if gold.dtype != torch.float32 else gold.view(torch.int32))


def test_fully_masked_rows_are_nan_in_reference():
    case = next(c for c in META["cases"] if c["name"] == "bf16_fully_masked_batch")
    gold = _golden_tensor(case).float()
    assert torch.isnan(gold[1]).all() and not torch.isnan(gold[0]).any()


@pytest.mark.parametrize("causal", [False, True])
def test_row_blocked_oracle_equals_dense(causal):
    gen = torch.Generator().manual_seed(3)
    q, k, v = (torch.randn((2, 2, 200, 64), generator=gen).bfloat16() for _ in range(3))
    mask = torch.arange(200)[None, :] < torch.tensor([200, 150])[:, None]
    dense = reference_attention(q, k, v, mask, causal, 0.125)
    blocked = reference_attention_blocked(q, k, v, mask, causal, 0.125, rows_per_block=64)
    torch.testing.assert_close(blocked.float(), dense.float(), rtol=0, atol=0)
    rows = reference_attention_rows(q, k, v, mask, causal, 0.125, 37, 101)
    torch.testing.assert_close(rows.float(), dense[:, :, 37:101].float(), rtol=0, atol=0)


def test_zero_masked_rows():
    out = torch.ones(2, 1, 4, 2)
    mask = torch.tensor([[True, True, False, False], [True, False, True, False]])
    z = zero_masked_rows(out, mask)
    assert z[0, 0, 2:].abs().sum() == 0 and z[1, 0, 1].abs().sum() == 0 and z[1, 0, 2].sum() == 2


def test_flop_counts_match_the_configuration_totals():
    # cfg2 137.4 GFLOP causal, north-star 2199.0 GFLOP, cfg4 8796 GFLOP
    assert abs(attention_flops(8, 16, 2048, 128, True) / 1e9 - 137.4) < 0.1
    assert abs(attention_flops(8, 16, 8192, 128, True) / 1e9 - 2199.0) < 0.1
    assert abs(attention_flops(1, 32, 32768, 128, True) / 1e9 - 8796.1) < 0.1
    assert attention_flops(2, 1, 10, 8, False, valid_lengths=[3, 4]) == 4 * 8 * (9 + 16)
