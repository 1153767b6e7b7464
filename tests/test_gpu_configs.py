"""Kernel parity at the BASELINE configurations' full sizes, and against the
reference's own golden outputs.

The kernel runs the whole configuration on the GPU; the CPU oracle (the
reference's operation order) checks every (batch, head) where that takes
seconds, and otherwise sampled heads and query-row ranges through its
bounded row form (the reference's own long-sequence tests sample rows the same
way, test/test_triton_fused_attention.py:612-635).  Inputs follow the
reference's generator (seeded torch.randn in fp32, cast to bf16).

Tolerance: max-abs <= 2e-2 and mean-abs <= 2e-3 (``parity.py``).
"""

import json
from pathlib import Path

import numpy as np
import pytest
import torch

from b200_attention import b200_fused_attention, read_device_errors
from oracle.reference_attention import reference_attention, reference_attention_rows, zero_masked_rows
from parity import assert_close, seeded_qkv
from tests_golden_io import load_case_inputs

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
GOLDEN = Path(__file__).resolve().parent / "golden"


def _kernel(q, k, v, mask, causal, zero_q=False):
    out = b200_fused_attention(q.to(DEV), k.to(DEV), v.to(DEV),
                               None if mask is None else mask.to(DEV), causal,
                               zero_masked_queries=zero_q)
    torch.cuda.synchronize()
    assert read_device_errors(DEV) == 0
    return out.cpu()


def test_cfg1_full():
    q, k, v = seeded_qkv((2, 8, 512, 64), torch.bfloat16, 1234)
    assert_close(_kernel(q, k, v, None, True), reference_attention(q, k, v, None, True, 0.125), "cfg1")


def test_cfg2_full():
    shape = (8, 16, 2048, 128)
    q, k, v = seeded_qkv(shape, torch.bfloat16, 1234)
    out = _kernel(q, k, v, None, True)
    for b in range(shape[0]):
        ref = reference_attention(q[b:b + 1], k[b:b + 1], v[b:b + 1], None, True, 128 ** -0.5)
        assert_close(out[b:b + 1], ref, f"cfg2 batch {b}")


def test_cfg3_key_padded_every_batch_entry():
    B, H, S, D = 16, 32, 4096, 128
    q, k, v = seeded_qkv((B, H, S, D), torch.bfloat16, 1234)
    gen = torch.Generator("cpu").manual_seed(1234 + 7)
    lengths = torch.randint(S // 4, S + 1, (B,), generator=gen)
    mask = torch.arange(S)[None, :] < lengths[:, None]
    out = _kernel(q, k, v, mask, False, zero_q=True)
    # one head of every batch entry (every valid length), heads spread over 0..H-1
    for b in range(B):
        h = (b * 7) % H
        sl = (slice(b, b + 1), slice(h, h + 1))
        ref = reference_attention(q[sl], k[sl], v[sl], mask[b:b + 1], False, D ** -0.5)
        ref = zero_masked_rows(ref, mask[b:b + 1])
        assert_close(out[sl], ref, f"cfg3 b={b} L={int(lengths[b])} h={h}")


@pytest.mark.parametrize("name,shape", [("ns", (8, 16, 8192, 128)), ("cfg4", (1, 32, 32768, 128)),
                                        ("s100k", (1, 1, 100000, 128))])
def test_long_causal_sampled_rows(name, shape):
    B, H, S, D = shape
    q, k, v = seeded_qkv(shape, torch.bfloat16, 1234)
    out = _kernel(q, k, v, None, True)
    pairs = [(0, 0), (B - 1, H - 1)]
    rows = [(0, 256), (S // 2 - 128, S // 2 + 128), (S - 256, S)]
    for b, h in pairs:
        sl = (slice(b, b + 1), slice(h, h + 1))
        for r0, r1 in rows:
            ref = reference_attention_rows(q[sl], k[sl], v[sl], None, True, D ** -0.5, r0, r1)
            assert_close(out[sl][:, :, r0:r1], ref, f"{name} b={b} h={h} rows {r0}:{r1}")


def test_kernel_against_reference_golden_outputs():
    """The reference's own outputs (tests/golden, produced by importing the
    reference) for every case the kernel covers (bf16/fp16 at D 64/128, fp32 at
    D 64)."""
    meta = json.loads((GOLDEN / "attention_cases.json").read_text())
    arrays = np.load(GOLDEN / "attention_cases.npz")
    checked = 0
    for case in meta["cases"]:
        if case["shape"][3] not in (64, 128) or (case["dtype"] == "float32" and case["shape"][3] > 64):
            continue
        q, k, v, mask = load_case_inputs(case)
        out = _kernel(q, k, v, mask, case["causal"])
        keep = case["keep_heads"]
        if keep:
            out = out[:, :keep]
        dt = {"bfloat16": torch.bfloat16, "float16": torch.float16,
              "float32": torch.float32}[case["dtype"]]
        golden = torch.from_numpy(arrays[case["name"]].copy())
        golden = golden if dt == torch.float32 else golden.view(dt)
        assert_close(out, golden, case["name"])
        checked += 1
    assert checked >= 8


def test_autograd_routes_to_the_exact_path_on_cuda():
    """With autograd requested, the planner picks the organiser's exact order
    (as the reference planner does) and gradients flow."""
    from b200_attention.attention_dispatch import AttentionMode
    from b200_attention.modules import B200FusedSelfAttention

    torch.manual_seed(0)
    mod = B200FusedSelfAttention(256, 4).to(DEV, torch.bfloat16)
    x = torch.randn(2, 64, 256, device=DEV, dtype=torch.bfloat16, requires_grad=True)
    out = mod(x, None, causal=True)
    _, plan = mod._attention_plan(x, True, True)
    assert plan.mode == AttentionMode.EXACT_REFERENCE
    out.float().sum().backward()
    assert x.grad is not None and torch.isfinite(x.grad.float()).all()


def test_bench_line_carries_the_contract_fields():
    """bench.py on one GPU (short cfg1 run): the JSON line has the fields the
    benchmark contract asks for, counted launches and a clock record."""
    import subprocess
    import sys

    root = Path(__file__).resolve().parents[1]
    proc = subprocess.run([sys.executable, str(root / "bench.py"), "--workload", "cfg1", "--steps", "16",
                           "--warmup", "3", "--cpu-budget", "0.5", "--e2e-steps", "3"],
                          capture_output=True, text=True, timeout=600, cwd=root)
    assert proc.returncode == 0, proc.stderr[-3000:]
    d = json.loads([l for l in proc.stdout.splitlines() if l.startswith("{")][-1])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
                "roofline", "cpu_baseline", "e2e", "gpu_launches", "clocks"):
        assert key in d, key
    r = d["roofline"]
    assert r["bound"] == "hbm" and r["unit"] == "GB/s" and 0 < r["frac"] < 1.5
    assert r["tensor"]["unit"] == "TFLOP/s" and r["traffic_source"]["file"].startswith("profiles/")
    assert d["gpu_launches"] == 16 and d["validation"]["device_errors"] == 0
    assert d["e2e"]["h2d_bytes_per_step"] > 0 and d["e2e"]["d2h_bytes_per_step"] > 0
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
