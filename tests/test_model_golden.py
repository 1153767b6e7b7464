"""Model-level parity pinned to the reference itself, on CPU.

``tests/golden/model_cases.*`` hold what the reference's own
``BaselineTransformer`` (torch_transformer_benchmark.py:126-171) computed on
CPU for a 2-layer decoder (fp32, bf16 and fp16; causal and key-padded), block
by block and for the whole model.  On a CPU device this package's decoder plans
the exact operation order for every layer, so its blocks and its output must
equal the reference's bit for bit; so must the restated baseline the GPU tests
use as their reference (``tests/e2e_models.py``).
"""

import json
from pathlib import Path

import numpy as np
import pytest
import torch

from b200_attention.transformer import Decoder, DecoderConfig
from e2e_models import OracleSelfAttention
from tests_golden_io import DTYPES, model_case_inputs, seeded_state_dict

GOLDEN = Path(__file__).resolve().parent / "golden"
META = json.loads((GOLDEN / "model_cases.json").read_text())
CASES = {c["name"]: c for c in META["cases"]}


def golden_tensor(name: str, dtype: torch.dtype) -> torch.Tensor:
    with np.load(GOLDEN / "model_cases.npz") as z:
        arr = z[name]
    t = torch.from_numpy(arr.copy())
    return t if dtype == torch.float32 else t.view(dtype)


def build(case, attention_cls=None) -> Decoder:
    cfg = DecoderConfig(case["batch"], case["seq_len"], case["d_model"], case["num_heads"],
                        case["ffn_dim"], case["num_layers"], case["causal"])
    dtype = DTYPES[case["dtype"]]
    kw = {} if attention_cls is None else dict(attention_cls=attention_cls, model_scoped_plans=False)
    model = Decoder(cfg, **kw)
    model.load_state_dict(seeded_state_dict(model.state_dict(), case["weight_seed"], dtype),
                          strict=True)
    return model.to(dtype).eval()


@pytest.mark.parametrize("name", sorted(CASES))
@pytest.mark.parametrize("which", ["decoder", "restated_baseline"])
def test_cpu_model_equals_reference_bit_for_bit(name, which):
    case = CASES[name]
    dtype = DTYPES[case["dtype"]]
    model = build(case, None if which == "decoder" else OracleSelfAttention)
    x, mask = model_case_inputs(case)
    with torch.inference_mode():
        h = x
        for i, layer in enumerate(model.layers):
            h = layer(h, mask, case["causal"])
            assert torch.equal(h, golden_tensor(f"{name}.block{i}", dtype)), f"block {i}"
        out = model(x, mask)
    assert torch.equal(out, golden_tensor(f"{name}.out", dtype))


def test_fixture_covers_the_dtypes_and_masks():
    assert {c["dtype"] for c in CASES.values()} == {"float32", "bfloat16", "float16"}
    assert any(c["padding_ratio"] is None for c in CASES.values())
    assert any((c["padding_ratio"] or 0) > 0 for c in CASES.values())
    assert any(not c["causal"] for c in CASES.values())
