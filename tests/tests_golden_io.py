"""Regenerate golden-case inputs from their seeds and check their digest."""

import hashlib

import torch

DTYPES = {"bfloat16": torch.bfloat16, "float16": torch.float16, "float32": torch.float32}


def load_case_inputs(case):
    shape = tuple(case["shape"])
    gen = torch.Generator("cpu").manual_seed(case["seed"])
    q, k, v = (torch.randn(shape, generator=gen, dtype=torch.float32).to(DTYPES[case["dtype"]])
               for _ in range(3))
    mask = None
    if case["lengths"] is not None:
        mask = torch.arange(shape[2])[None, :] < torch.tensor(case["lengths"])[:, None]
    h = hashlib.sha256()
    for t in (q, k, v):
        h.update(t.contiguous().view(torch.uint8).numpy().tobytes() if t.dtype != torch.float32
                 else t.contiguous().numpy().tobytes())
    if mask is not None:
        h.update(mask.numpy().tobytes())
    assert h.hexdigest() == case["input_sha256"], "seeded generator drifted from the fixture"
    return q, k, v, mask


def seeded_state_dict(template: dict, seed: int, dtype: torch.dtype) -> dict:
    """Deterministic weights for a model whose state dict has ``template``'s
    keys and shapes, independent of module order (keys in sorted order):
    linear weights N(0, 0.02), biases N(0, 0.02), LayerNorm weights
    1 + N(0, 0.1).  The reference model and this package's decoder share the
    organiser's parameter names, so one seed gives both the same weights."""
    gen = torch.Generator("cpu").manual_seed(seed)
    out = {}
    for key in sorted(template):
        shape = tuple(template[key].shape)
        noise = torch.randn(shape, generator=gen, dtype=torch.float32)
        is_norm_weight = key.endswith("weight") and "norm" in key.rsplit(".", 2)[-2]
        out[key] = (1.0 + 0.1 * noise if is_norm_weight else 0.02 * noise).to(dtype)
    return out


def model_digest(x: torch.Tensor, mask) -> str:
    h = hashlib.sha256()
    h.update(x.contiguous().view(torch.uint8).numpy().tobytes())
    if mask is not None:
        h.update(mask.contiguous().numpy().tobytes())
    return h.hexdigest()


def model_case_inputs(case):
    """Hidden states and key mask of a model case, made the way the reference
    harness's generate_random_case makes them (torch_transformer_benchmark.py:
    362-400): x ~ N(0, 1) drawn in the model dtype from a seeded CPU generator,
    valid lengths uniform in [round(S * (1 - padding_ratio)), S], padded rows
    of x zeroed; padding_ratio 0 gives an all-ones mask, None no mask."""
    B, S, d = case["batch"], case["seq_len"], case["d_model"]
    gen = torch.Generator("cpu").manual_seed(case["seed"])
    x = torch.randn(B, S, d, generator=gen, dtype=DTYPES[case["dtype"]])
    ratio = case["padding_ratio"]
    if ratio is None or ratio <= 0:
        mask = None if ratio is None else torch.ones(B, S, dtype=torch.bool)
    else:
        low = max(1, int(round(S * (1.0 - ratio))))
        lengths = torch.randint(low=low, high=S + 1, size=(B,), generator=gen)
        mask = torch.arange(S)[None, :] < lengths[:, None]
        x = x.masked_fill(~mask[..., None], 0)
    assert model_digest(x, mask) == case["input_sha256"], "seeded generator drifted from the fixture"
    return x, mask
