"""Shared parity helpers for the GPU tests (tolerances are stated here once).

Tolerance for bf16/fp16 outputs against the fp32-softmax PyTorch reference:
max-abs <= 2e-2 and mean-abs <= 2e-3.  The organiser's per-element OR rule
(|d| <= 2e-3 or |d| <= 2e-2 * |ref|, torch_transformer_benchmark.py:1-12) is
reported as the fraction of elements that fail it.
"""

from __future__ import annotations

import torch

MAX_ABS = 2e-2
MEAN_ABS = 2e-3
OR_ATOL = 2e-3
OR_RTOL = 2e-2


def seeded_qkv(shape, dtype, seed=1234, device="cpu"):
    """Q, K, V i.i.d. N(0,1) in fp32 from a seeded CPU generator, cast to dtype."""
    gen = torch.Generator("cpu").manual_seed(seed)
    q, k, v = (torch.randn(shape, generator=gen, dtype=torch.float32) for _ in range(3))
    return q.to(device=device, dtype=dtype), k.to(device=device, dtype=dtype), v.to(device=device, dtype=dtype)


def prefix_mask(batch, seq_len, lengths, device="cpu"):
    idx = torch.arange(seq_len)[None, :]
    return (idx < torch.tensor(lengths)[:, None]).to(device)


def compare(out: torch.Tensor, ref: torch.Tensor) -> dict:
    out = out.float().cpu()
    ref = ref.float().cpu()
    nan_out, nan_ref = torch.isnan(out), torch.isnan(ref)
    same_nan = bool(torch.equal(nan_out, nan_ref))
    finite = ~nan_ref
    diff = (out - ref).abs()[finite]
    refa = ref.abs()[finite]
    if diff.numel() == 0:
        return {"max_abs": 0.0, "mean_abs": 0.0, "or_fail_frac": 0.0, "same_nan": same_nan}
    or_fail = ~((diff <= OR_ATOL) | (diff <= OR_RTOL * refa))
    return {
        "max_abs": float(diff.max()),
        "mean_abs": float(diff.mean()),
        "or_fail_frac": float(or_fail.float().mean()),
        "same_nan": same_nan,
    }


def assert_close(out: torch.Tensor, ref: torch.Tensor, label: str = "") -> dict:
    r = compare(out, ref)
    assert r["same_nan"], f"{label}: NaN pattern differs {r}"
    assert r["max_abs"] <= MAX_ABS, f"{label}: max-abs {r}"
    assert r["mean_abs"] <= MEAN_ABS, f"{label}: mean-abs {r}"
    return r


def unit_in_last_place(ref: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """Unit in the last place of each element of ``ref`` in ``dtype``."""
    mant = {torch.bfloat16: 7, torch.float16: 10, torch.float32: 23}[dtype]
    mag = ref.float().abs().clamp_min(torch.finfo(dtype).tiny)
    return torch.exp2(torch.floor(torch.log2(mag)) - mant)


# A block's output is a 16-bit residual stream, rounded three times after the
# attention sublayer: x1 = round(x + attention), f = ffn(LayerNorm(x1)) rounded
# at each of its steps, out = round(x1 + f).  Two implementations whose
# attention differs in its last bits can differ by one unit of the stream's
# magnitude in x1, by up to two units where that flip passes through the
# LayerNorm and the FFN into f, and by one more in the final sum: four units in
# the last place of the row's largest magnitude.  (The reference block with an
# exact fp32 attention core reaches 1.5 units against the bf16 block at the
# end-to-end configuration, whose stream grows to |x| ~ 9, where one bf16 unit
# is 0.0625 -- above the 2e-2 of an attention output of magnitude < 2.)  The
# bound for a block's output is max(MAX_ABS, BLOCK_UNITS such units) per
# element, with the mean-abs bound unchanged.
BLOCK_UNITS = 4


def assert_block_close(out: torch.Tensor, ref: torch.Tensor, dtype: torch.dtype,
                       label: str = "") -> dict:
    """A decoder block's output against the reference block's: the mean-abs
    bound, the NaN pattern, and max(MAX_ABS, BLOCK_UNITS row units) per element."""
    r = compare(out, ref)
    assert r["same_nan"], f"{label}: NaN pattern differs {r}"
    assert r["mean_abs"] <= MEAN_ABS, f"{label}: mean-abs {r}"
    o, f = out.float().cpu(), ref.float().cpu()
    row_max = f.abs().nan_to_num(0.0).amax(dim=-1, keepdim=True)
    bound = torch.clamp(BLOCK_UNITS * unit_in_last_place(row_max, dtype), min=MAX_ABS)
    d = (o - f).abs().nan_to_num(0.0)
    assert bool((d <= bound).all()), f"{label}: worst {float((d - bound).max()):.3e} over the bound {r}"
    return r
