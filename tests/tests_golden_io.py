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
