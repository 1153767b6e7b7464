"""Model-level parity on the GPU against the reference's own BaselineTransformer.

The fixtures (``tests/golden/model_cases.*``) are the reference model's
outputs on CPU, block by block.  Here each block of this package's decoder --
its LayerNorms, attention and linear layers on the B200 kernels for 16-bit
inputs -- is fed the reference's output of the previous block, so every
block's error is measured on its own instead of compounded through the stack.

Tolerances (``parity.py``):

* the attention sublayer of each block (the projections, the attention kernel
  and the padded-row zeroing, fed the block's normalised input): north_star's
  max-abs <= 2e-2 and mean-abs <= 2e-3;
* each block's output, a 16-bit residual sum: mean-abs <= 2e-3 and, per
  element, max(2e-2, four units in the last place of the row's largest
  magnitude, ``parity.BLOCK_UNITS``) -- below that, two correct
  implementations differ by the rounding of the residual stream itself;
* the final LayerNorm of the reference's last block output: at most one unit
  in the last place of the reference value (16-bit; fp32 gets the absolute
  bound above);
* the whole model end to end is reported, and must be finite with the
  reference's NaN pattern.
"""

import pytest
import torch

from b200_attention.attention_dispatch import AttentionMode
from b200_attention.layernorm import b200_layer_norm
from parity import assert_block_close, assert_close, compare, unit_in_last_place
from test_model_golden import CASES, build, golden_tensor
from tests_golden_io import DTYPES, model_case_inputs

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


@pytest.mark.parametrize("name", sorted(CASES))
def test_gpu_blocks_match_reference_model(name):
    case = CASES[name]
    dtype = DTYPES[case["dtype"]]
    causal = case["causal"]
    model = build(case).to(DEV)
    x, mask = model_case_inputs(case)
    mask_d = None if mask is None else mask.to(DEV)
    with torch.inference_mode():
        prev = x.to(DEV)
        for i, layer in enumerate(model.layers):
            attn = layer.attention(layer.norm1(prev), mask_d, causal)
            if dtype != torch.float32:
                assert layer._fusable(prev), "the block must run on the fused kernels"
                assert layer.attention._plan_value[1].mode == AttentionMode.SM100_FUSED
            r_attn = assert_close(attn, golden_tensor(f"{name}.attn{i}", dtype),
                                  f"{name} attention {i}")
            out = layer(prev, mask_d, causal)
            ref = golden_tensor(f"{name}.block{i}", dtype)
            r = assert_block_close(out, ref, dtype, f"{name} block {i}")
            print(f"\n{name} layer {i}: attention {r_attn}\n  block {r}")
            prev = ref.to(DEV)

        fn = model.final_norm
        if dtype == torch.float32:
            final = fn(prev)
        else:
            final = b200_layer_norm(prev, fn.weight, fn.bias, fn.eps)
        if mask_d is not None:
            final = final.masked_fill(~mask_d[..., None], 0)
        ref = golden_tensor(f"{name}.out", dtype)
        if dtype == torch.float32:
            # fp32 on both sides, reduced in different orders: x - mean cancels
            # near zero, so the bound is north_star's absolute one
            assert_close(final, ref, f"{name} final norm")
        else:
            d = (final.float().cpu() - ref.float()).abs()
            assert bool((d <= unit_in_last_place(ref, dtype)).all()), float(d.max())

        whole = model(x.to(DEV), mask_d)
        torch.cuda.synchronize()
    r = compare(whole, ref)
    print(f"{name} whole model: {r}")
    finite = ~torch.isnan(ref.float())
    assert r["same_nan"] and bool(torch.isfinite(whole.float().cpu()[finite]).all())
