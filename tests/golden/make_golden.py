"""Generate the golden fixtures from the reference itself (run in the build container).

    python tests/golden/make_golden.py --reference /path/to/reference

Writes, next to this script:

* ``attention_cases.json`` + ``attention_cases.npz`` — outputs of the
  reference's public operator ``triton_fused_attention`` on CPU tensors, which
  routes to its ``_reference_attention`` (model/triton_fused_attention.py:
  1906-1925, 1256-1285), for seeded inputs.  Inputs are regenerated from the
  seed by the tests; a SHA-256 of the input bytes guards against generator drift.
* ``planner_plans.json`` — the reference planner's plans
  (model/attention_dispatch.py:563) for the reference's 14 published shapes
  (tools/benchmark_shape_matrix.py) x dtype x device capability.
* ``model_cases.json`` + ``model_cases.npz`` — the reference's own
  ``BaselineTransformer`` (torch_transformer_benchmark.py:126-171) on CPU, with
  weights from ``tests_golden_io.seeded_state_dict`` and hidden states from the
  reference harness's ``generate_random_case`` (:362-400): for every block
  (fed the previous block's reference output) its attention sublayer's output
  and its own output, and the output of the whole model.

The reference is imported read-only; nothing of it is copied.  The fixtures are
what the reference computed, which is what the oracle must reproduce.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent

# (name, shape [B,H,S,D], dtype, causal, valid lengths or None, seed)
CASES = [
    ("bf16_causal_s64_d64", (1, 2, 64, 64), "bfloat16", True, None, 11),
    ("bf16_full_s130_d128", (2, 2, 130, 128), "bfloat16", False, None, 12),
    ("fp16_causal_mask_s257_d64", (2, 2, 257, 64), "float16", True, [257, 100], 13),
    ("bf16_causal_mask_s33_d128", (1, 1, 33, 128), "bfloat16", True, [20], 14),
    ("bf16_single_token_d128", (2, 2, 1, 128), "bfloat16", True, None, 15),
    ("bf16_fully_masked_batch", (2, 1, 70, 64), "bfloat16", False, [70, 0], 16),
    ("bf16_full_mask_s300_d128", (3, 2, 300, 128), "bfloat16", False, [300, 257, 1], 17),
    ("fp32_causal_s96_d64", (2, 1, 96, 64), "float32", True, None, 18),
    # configs[0] shape (B=2 H=8 S=512 D=64 causal, seed 1234) in the GPU dtype;
    # stored for heads 0-1 of each batch entry to keep the fixture small
    ("cfg1_bf16_causal_heads01", (2, 8, 512, 64), "bfloat16", True, None, 1234),
]
KEEP_HEADS = {"cfg1_bf16_causal_heads01": 2}

DTYPES = {"bfloat16": torch.bfloat16, "float16": torch.float16, "float32": torch.float32}

# Model cases: a 2-layer pre-LN decoder with the end-to-end configuration's
# head size (d_model 128, 2 heads of 64, FFN 512), B 2 x S 64.
# (name, dtype, causal, padding_ratio, seed); padding_ratio 0 gives the
# harness's all-ones mask, None no mask at all.
MODEL_SHAPE = dict(batch=2, seq_len=64, d_model=128, num_heads=2, ffn_dim=512, num_layers=2)
MODEL_WEIGHT_SEED = 4321
MODEL_CASES = [
    ("fp32_causal", "float32", True, 0.0, 1234),
    ("bf16_causal_nomask", "bfloat16", True, None, 1236),
    ("bf16_full_padded", "bfloat16", False, 0.5, 1237),
    ("fp16_causal_padded", "float16", True, 0.25, 1238),
]


def make_model_cases(reference_module):
    """Per-block and whole-model outputs of the reference's BaselineTransformer."""
    from tests_golden_io import model_digest, seeded_state_dict

    tb = reference_module
    meta, arrays = [], {}
    for name, dtype_name, causal, padding, seed in MODEL_CASES:
        dtype = DTYPES[dtype_name]
        cfg = tb.TransformerConfig(MODEL_SHAPE["batch"], MODEL_SHAPE["seq_len"],
                                   MODEL_SHAPE["d_model"], MODEL_SHAPE["num_heads"],
                                   MODEL_SHAPE["ffn_dim"], MODEL_SHAPE["num_layers"], causal)
        model = tb.BaselineTransformer(cfg)
        model.load_state_dict(seeded_state_dict(model.state_dict(), MODEL_WEIGHT_SEED, dtype))
        model = model.to(dtype).eval()
        x, mask = tb.generate_random_case(cfg, torch.device("cpu"), dtype, seed,
                                          0.0 if padding is None else padding, 1.0)
        if padding is None:
            mask = None
        with torch.inference_mode():
            h = x
            for i, layer in enumerate(model.layers):
                # the attention sublayer alone (the part the attention kernel
                # computes, with its projections), then the whole block
                arrays[f"{name}.attn{i}"] = to_bits(layer.attention(layer.norm1(h), mask, causal))
                h = layer(h, mask, causal)
                arrays[f"{name}.block{i}"] = to_bits(h)
            arrays[f"{name}.out"] = to_bits(model(x, mask))
        meta.append({"name": name, "dtype": dtype_name, "causal": causal, "padding_ratio": padding,
                     "seed": seed, **MODEL_SHAPE, "weight_seed": MODEL_WEIGHT_SEED,
                     "lengths": None if mask is None else mask.sum(1).tolist(),
                     "input_sha256": model_digest(x, mask)})
    np.savez_compressed(HERE / "model_cases.npz", **arrays)
    (HERE / "model_cases.json").write_text(json.dumps(
        {"torch": torch.__version__,
         "source": "reference BaselineTransformer (torch_transformer_benchmark.py) on CPU; "
                   "inputs from its generate_random_case",
         "cases": meta}, indent=1) + "\n")
    return len(meta)


def make_inputs(shape, dtype_name, lengths, seed):
    """Q, K, V ~ N(0,1) fp32 from a seeded CPU generator, cast (reference
    generator convention, torch_transformer_benchmark.py:362-400)."""
    gen = torch.Generator("cpu").manual_seed(seed)
    q, k, v = (torch.randn(shape, generator=gen, dtype=torch.float32).to(DTYPES[dtype_name])
               for _ in range(3))
    mask = None
    if lengths is not None:
        mask = torch.arange(shape[2])[None, :] < torch.tensor(lengths)[:, None]
    return q, k, v, mask


def input_digest(q, k, v, mask) -> str:
    h = hashlib.sha256()
    for t in (q, k, v):
        h.update(t.contiguous().view(torch.uint8).numpy().tobytes() if t.dtype != torch.float32
                 else t.contiguous().numpy().tobytes())
    if mask is not None:
        h.update(mask.numpy().tobytes())
    return h.hexdigest()


def to_bits(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.float32:
        return t.contiguous().numpy()
    return t.contiguous().view(torch.int16).numpy()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="checkout of the reference repository")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    sys.path.insert(0, str(HERE.parent))  # tests/ (tests_golden_io)
    import torch_transformer_benchmark
    from model.attention_dispatch import AttentionModelSpec, AttentionRuntime, select_attention_stack_plan
    from model.triton_fused_attention import triton_fused_attention
    from tools.benchmark_shape_matrix import ANNOUNCED_CASES

    meta, arrays = [], {}
    for name, shape, dtype, causal, lengths, seed in CASES:
        q, k, v, mask = make_inputs(shape, dtype, lengths, seed)
        out = triton_fused_attention(q, k, v, mask, causal, None)
        keep = KEEP_HEADS.get(name)
        if keep:
            out = out[:, :keep]
        arrays[name] = to_bits(out)
        meta.append({"name": name, "shape": list(shape), "dtype": dtype, "causal": causal,
                     "lengths": lengths, "seed": seed, "keep_heads": keep,
                     "input_sha256": input_digest(q, k, v, mask)})
    np.savez_compressed(HERE / "attention_cases.npz", **arrays)
    (HERE / "attention_cases.json").write_text(json.dumps(
        {"torch": torch.__version__, "source": "reference triton_fused_attention on CPU",
         "cases": meta}, indent=1) + "\n")

    plans = []
    for case in ANNOUNCED_CASES:
        spec = AttentionModelSpec(case.batch_size, case.seq_len, case.d_model, case.heads,
                                  case.ffn_dim, case.layers, case.causal)
        for dtype in ("float16", "bfloat16", "float32"):
            for cap in ((12, 0), (10, 0), (9, 0)):
                rt = AttentionRuntime(case.batch_size, case.seq_len, case.d_model, dtype, "cuda",
                                      cap, False, case.causal)
                for scope in ("model", "standalone"):
                    sp = select_attention_stack_plan(spec, rt, scope)
                    plans.append({
                        "case": case.case_id,
                        "spec": [case.batch_size, case.seq_len, case.d_model, case.heads,
                                 case.ffn_dim, case.layers, case.causal],
                        "dtype": dtype, "capability": list(cap), "scope": scope,
                        "execution": sp.execution,
                        "layers": [{"mode": p.mode.value, "family": p.family.value,
                                    "reason": p.reason.value if p.reason else None,
                                    "explanation": p.explanation,
                                    "launch": None if p.launch is None else {
                                        f: getattr(p.launch, f) for f in
                                        ("block_m", "block_n", "num_warps", "num_stages",
                                         "query_block_size", "output_layout")}}
                                   for p in sp.layers],
                    })
    (HERE / "planner_plans.json").write_text(json.dumps(plans, indent=0) + "\n")
    n_models = make_model_cases(torch_transformer_benchmark)
    print(f"wrote {len(meta)} attention cases, {len(plans)} plans and {n_models} model cases")


if __name__ == "__main__":
    main()
