#!/usr/bin/env python3
"""Benchmark of the sm_100a fused attention forward (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload cfg4]
    python bench.py --impl reference ...      # reference's CPU attention path
    python bench.py --impl torch-dense ...    # yardstick: the reference's dense path on this GPU

A step is one attention forward over one batch of the workload (one kernel
launch).  ``value`` is whole-job TFLOP/s with inputs resident in HBM; ``e2e``
is the same metric through the public operator with pinned host buffers and
the host<->device copies inside the timed region.  Multi-GPU runs use one
process per GPU (torchrun); each rank owns an independent (batch x head)
shard, there is no collective on the data path, and the time is the max over
ranks.  Inputs rotate over several buffers whose total exceeds the 126 MB L2.

FLOPs follow the algorithmic count 4*B*H*S^2*D (QK^T and PV), halved for
causal; for the key-padded workload only valid (query, key) pairs count,
4*H*D*sum(L_b^2), since padded query blocks are skipped.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for _p in (ROOT / "techjam-kernel_b200", ROOT):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

METRIC = "fused-attn fwd TFLOP/s & % bf16 tensor peak at 1/2/4/8 B200; vs CPU ms"
UNIT = "TFLOP/s"
L2_BYTES = 126 * 1024 * 1024
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}

# BASELINE configs.  The default workload is configs[3] (cfg4), the largest
# configuration that fits one GPU at N = 1 (all 32 heads; 4 heads per GPU at
# N = 8); "ns" is the north-star shape.
WORKLOADS = {
    "cfg1": dict(B=2, H=8, S=512, D=64, causal=True, masked=False, shard="batch"),
    # configs[0] in its own dtype: fp32 inputs on the fp32 instance (TF32 products)
    "cfg1f32": dict(B=2, H=8, S=512, D=64, causal=True, masked=False, shard="batch",
                    dtype="float32"),
    "cfg2": dict(B=8, H=16, S=2048, D=128, causal=True, masked=False, shard="batch"),
    "cfg3": dict(B=16, H=32, S=4096, D=128, causal=False, masked=True, shard="batch"),
    "cfg4": dict(B=1, H=32, S=32768, D=128, causal=True, masked=False, shard="heads"),
    "ns": dict(B=8, H=16, S=8192, D=128, causal=True, masked=False, shard="batch"),
    # end-to-end: 12-layer pre-LN decoder, d_model 1024, FFN 4096, vocab 32000;
    # global batch 8 split over the ranks (data parallel)
    "cfg5": dict(B=8, H=16, S=2048, D=64, causal=True, masked=False, shard="batch_split",
                 layers=12, d_model=1024, ffn=4096, vocab=32000),
    # context parallelism: one long causal sequence sharded (zigzag) over the
    # ranks, K/V passed around a ring; strong scaling
    "cp": dict(B=1, H=8, S=131072, D=128, causal=True, masked=False, shard="sequence",
               kind="context_parallel"),
    # the row softmax over materialised scores (the reference's unfused seam,
    # model/triton_softmax.py) at cfg2's score shape [8, 16, 2048, 2048]
    "sm2": dict(B=8, H=16, S=2048, D=128, causal=True, masked=False, shard="batch",
                kind="softmax"),
    # the reference's only published attention timing (fp16 two-pass tiled
    # attention, docs/TECH_REPORT.md:98-111): 0.590592 ms on an RTX 5070 Ti
    "tr": dict(B=64, H=4, S=1024, D=32, causal=True, masked=False, shard="batch", dtype="float16",
               published_ms=0.590592, published_hw="RTX 5070 Ti (sm_120), fp16 two-pass Triton"),
}


def cfg_dtype(cfg: dict):
    import torch

    return getattr(torch, cfg.get("dtype", "bfloat16"))


def dtype_tag(cfg: dict) -> str:
    return {"bfloat16": "bf16", "float16": "fp16", "float32": "fp32 (tf32 products)"}[
        cfg.get("dtype", "bfloat16")]


def load_peaks() -> tuple[dict, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        return json.loads(path.read_text()), "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def algorithmic_bytes(cfg: dict, batch: int, heads: int, lengths: list[int] | None) -> float:
    """Minimum HBM bytes of one launch: Q, K and V read once and O written once
    (for key-padded batches only the valid query and key rows are read, the
    whole output is written), plus the key mask."""
    S, D = cfg["S"], cfg["D"]
    elem = 4 if cfg.get("dtype") == "float32" else 2
    if lengths is not None:
        rows_read = heads * 3 * sum(lengths)
        return float(elem * D * (rows_read + batch * heads * S) + batch * S)
    return float(4 * batch * heads * S * D * elem)


def roofline(flop: float, nbytes: float, launch_ms: float, peaks: dict, peak_src: str,
             traffic, traffic_source) -> dict:
    """Roofline of one launch.  The bound is the roof the arithmetic intensity
    puts the kernel under: tensor when FLOP/byte is above the ridge (measured
    bf16 peak / measured HBM bandwidth), HBM otherwise; both fractions are
    reported."""
    tflops = flop / (launch_ms * 1e-3) / 1e12
    gbs = nbytes / (launch_ms * 1e-3) / 1e9
    ai = flop / nbytes
    ridge = peaks["bf16_tflops"] * 1e12 / (peaks["hbm_gbs"] * 1e9)
    tensor = {"achieved": tflops, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
              "frac": tflops / peaks["bf16_tflops"]}
    hbm = {"achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": gbs / peaks["hbm_gbs"]}
    main = tensor if ai >= ridge else hbm
    return {
        "bound": "tensor" if ai >= ridge else "hbm", **main, "traffic": traffic,
        "algorithmic_bytes": nbytes, "flop": flop, "arithmetic_intensity": ai, "ridge": ridge,
        "tensor": tensor, "hbm": hbm, "avg_launch_ms": launch_ms,
        "peak_source": f"{peak_src} bf16_tflops (burst, kernel timed alone) and hbm_gbs",
        "traffic_source": traffic_source,
    }


def stored_traffic(name: str, scale: float = 1.0):
    """DRAM bytes per launch from a committed ncu capture (profiles/), scaled
    to this rank's share of the launch, with the capture's provenance."""
    prof = ROOT / "profiles" / name
    if not prof.exists():
        return None, None
    data = json.loads(prof.read_text())
    traffic = data.get("dram_bytes_per_launch")
    source = {"file": f"profiles/{name}", "commit": data.get("captured_at_commit"),
              "workload": data.get("workload")}
    return (traffic * scale if traffic is not None else None), source


def valid_lengths(cfg: dict, seed: int) -> list[int] | None:
    """Per-sequence valid lengths ~ U{S/4..S} from the seed (cfg3)."""
    if not cfg["masked"]:
        return None
    import torch

    gen = torch.Generator("cpu").manual_seed(seed + 7)
    S = cfg["S"]
    return torch.randint(S // 4, S + 1, (cfg["B"],), generator=gen).tolist()


def flops_for(cfg: dict, batch: int, heads: int, lengths: list[int] | None) -> float:
    S, D = cfg["S"], cfg["D"]
    if lengths is not None:
        return 4.0 * heads * D * float(sum(L * L for L in lengths))
    f = 4.0 * batch * heads * S * S * D
    return f / 2 if cfg["causal"] else f


def shard_for(cfg: dict, world: int, rank: int) -> tuple[int, int, str]:
    """(batch, heads) this rank processes and the scaling kind.

    Weak scaling: every rank runs the full per-GPU workload (a data-parallel
    job of N x B sequences).  Strong scaling (cfg4): the H heads are split in
    contiguous ranges over the ranks (4 heads per GPU at N = 8)."""
    if cfg["shard"] == "heads":
        H = cfg["H"]
        lo = (H * rank) // world
        hi = (H * (rank + 1)) // world
        return cfg["B"], hi - lo, "strong"
    if cfg["shard"] == "batch_split":
        B = cfg["B"]
        return (B * (rank + 1)) // world - (B * rank) // world, cfg["H"], "strong"
    return cfg["B"], cfg["H"], "weak"


class ClockSampler:
    """Samples SM clock and throttle reasons via NVML while the timed region runs."""

    REASONS = {
        0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
        0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown", 0x2: "applications_clocks_setting",
    }

    def __init__(self, device_index: int, interval_s: float = 0.005):
        self.interval = interval_s
        self.samples: list[tuple[int, int]] = []
        self.max_mhz = None
        self.ok = False
        self._stop = threading.Event()
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nvml = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            self._nvml = None

    def _run(self):
        n = self._nvml
        while not self._stop.is_set():
            try:
                mhz = n.nvmlDeviceGetClockInfo(self._h, n.NVML_CLOCK_SM)
                reasons = n.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                self.samples.append((mhz, reasons))
            except Exception:
                pass
            time.sleep(self.interval)

    def __enter__(self):
        if self.ok:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *exc):
        if self.ok:
            self._stop.set()
            self._t.join()

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0,
                    "source": "nvml" if self.ok else "unavailable"}
        mhz = [s[0] for s in self.samples]
        mask = 0
        for _, r in self.samples:
            mask |= r
        reasons = sorted(name for bit, name in self.REASONS.items() if mask & bit)
        return {"sm_mhz": statistics.median(mhz), "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(mhz), "source": "nvml"}


class CpuReference:
    """The reference's CPU attention path timed on a bounded slice of the workload.

    The timed call is the oracle's restatement of _reference_attention (torch CPU
    ops in the reference's operation order, model/triton_fused_attention.py:1256-1285)
    with all host threads.  The slice is one batch entry and enough heads for
    ~0.1-0.5 s per call; for S > 8192 it is the last 512 query rows of one head
    (the heaviest causal rows) through the bounded row form.
    """

    def __init__(self, cfg: dict, seed: int = 1234):
        import torch

        from oracle import reference_attention as ora

        torch.set_num_threads(os.cpu_count() or 1)
        self.torch, self.ora = torch, ora
        S, D, causal = cfg["S"], cfg["D"], cfg["causal"]
        self.S, self.D, self.causal = S, D, causal
        heads = max(1, min(cfg["H"], int(2 ** 31 // (S * S * 12))))
        gen = torch.Generator("cpu").manual_seed(seed)
        self.q, self.k, self.v = (torch.randn((1, heads, S, D), generator=gen).to(cfg_dtype(cfg))
                                  for _ in range(3))
        lengths = valid_lengths(cfg, seed)
        self.mask = None
        self.rows = None
        if S > 8192:
            self.rows = (S - 512, S)
            visible = sum((r + 1) if causal else S for r in range(*self.rows))
            self.flop = 4.0 * heads * D * visible
        elif lengths is not None:
            L = lengths[0]
            self.mask = torch.arange(S)[None, :] < L
            self.flop = 4.0 * heads * D * L * L
        else:
            self.flop = flops_for(cfg, 1, heads, None)
        self.desc = (f"oracle.reference_attention (torch CPU, {dtype_tag(cfg)}, reference op order) on "
                     f"[1,{heads},{S},{D}] causal={causal}"
                     + (f" rows {self.rows[0]}..{self.rows[1] - 1}" if self.rows else "")
                     + (f" key-mask L={lengths[0]}" if self.mask is not None else "")
                     + f"; {self.flop / 1e9:.2f} GFLOP per sample")
        self.call()  # warm-up

    def call(self) -> float:
        t0 = time.perf_counter()
        if self.rows is not None:
            self.ora.reference_attention_rows(self.q, self.k, self.v, None, self.causal,
                                              self.D ** -0.5, *self.rows)
        else:
            self.ora.reference_attention(self.q, self.k, self.v, self.mask, self.causal, self.D ** -0.5)
        return time.perf_counter() - t0

    def measure(self, budget_s: float, min_reps: int = 1, full_flop: float | None = None) -> dict:
        times = []
        while sum(times) < budget_s or len(times) < min_reps:
            times.append(self.call())
        med = statistics.median(times)
        rate = self.flop / med
        out = {"value": rate / 1e12, "unit": UNIT,
               "cores": self.torch.get_num_threads(), "kind": "port",
               "ms_per_sample": med * 1e3, "sample": f"{len(times)} reps of " + self.desc}
        if full_flop:
            # the metric's "vs CPU ms": the whole step on the CPU at the sampled rate
            out["ms_per_step_extrapolated"] = full_flop / rate * 1e3
            out["sample"] += (f"; full step extrapolated at the sampled FLOP rate: "
                              f"{full_flop / 1e12:.3f} TFLOP / {rate / 1e12:.3f} TFLOP/s")
        return out


def run_reference_softmax_arm(args, cfg: dict, world: int) -> int:
    """Reference arm of the softmax workload: the reference's softmax stage
    (oracle.reference_softmax, torch CPU ops in its order) on host cores, on one
    batch entry of the score tensor, in the GPU arm's unit (GB/s)."""
    import torch

    from oracle.reference_attention import reference_softmax

    torch.set_num_threads(os.cpu_count() or 1)
    B, H, _ = shard_for(cfg, 1, 0)
    S, D = cfg["S"], cfg["D"]
    dtype = cfg_dtype(cfg)
    elem = torch.finfo(dtype).bits // 8
    heads = max(1, min(H, int(2 ** 31 // (S * S * 12))))
    gen = torch.Generator("cpu").manual_seed(args.seed)
    scores = (4 * torch.randn((1, heads, S, S), generator=gen)).to(dtype)
    for _ in range(args.warmup):
        reference_softmax(scores, None, D ** -0.5, cfg["causal"])
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        reference_softmax(scores, None, D ** -0.5, cfg["causal"])
        times.append(time.perf_counter() - t0)
    sec = statistics.median(times)
    sample_bytes = 2.0 * heads * S * S * elem
    value = sample_bytes / sec / 1e9
    desc = (f"oracle.reference_softmax (torch CPU, reference op order) on [1,{heads},{S},{S}] "
            f"{dtype_tag(cfg)}; {args.steps} timed reps")
    print(json.dumps({
        "impl": "reference", "metric": "row softmax over materialised attention scores, GB/s",
        "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 2.0 * B * H * S * S * elem / (value * 1e9) * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": dtype_tag(cfg),
        "data": "synthetic (seeded 4 * N(0,1) scores)",
        "config": {"workload": args.workload, "B": B, "H": H, "S": S, "causal": cfg["causal"],
                   "impl_path": "oracle.reference_softmax on host CPU cores"},
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": torch.get_num_threads(),
                         "kind": "port", "sample": desc},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)
    return 0


def run_reference_arm(args, cfg: dict, rank: int, world: int) -> int:
    """Reference arm: the reference's CPU attention on host cores, rank 0 only."""
    if rank != 0:
        return 0
    if cfg.get("kind") == "softmax":
        return run_reference_softmax_arm(args, cfg, world)
    ref = CpuReference(cfg, args.seed)
    for _ in range(args.warmup):
        ref.call()
    times = [ref.call() for _ in range(args.steps)]
    ms = statistics.median(times) * 1e3
    value = ref.flop / (ms * 1e-3) / 1e12
    B, H, _ = shard_for(cfg, 1, 0)
    full_flop = flops_for(cfg, B, H, valid_lengths(cfg, args.seed))
    line = {
        "impl": "reference",
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak" if cfg["shard"] != "heads" else "strong",
        "vs_baseline": None, "dtype": dtype_tag(cfg), "data": "synthetic (seeded torch.randn N(0,1))",
        "config": {"workload": args.workload, **{k: cfg[k] for k in ("B", "H", "S", "D", "causal")},
                   "impl_path": "oracle.reference_attention on host CPU cores"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": ref.torch.get_num_threads(),
                         "kind": "port", "sample": f"{args.steps} timed reps of " + ref.desc
                         + f"; full step extrapolated at the sampled FLOP rate",
                         "ms_per_step_extrapolated": full_flop / (value * 1e12) * 1e3},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def dense_torch_attention(q, k, v, mask, causal: bool, scale: float, max_score_bytes: int):
    """The reference's own B200 path in torch CUDA ops: _reference_attention
    (model/triton_fused_attention.py:1256-1285), which the reference's planner
    selects on capability 10.x (model/attention_dispatch.py:362-363).  QK^T in
    the input dtype, x scale in dtype, causal triu(1) and key mask to -inf, fp32
    softmax, cast, PV.  Heads are processed in chunks so the fp32 score tensor
    stays under max_score_bytes.  Returns [B, H, S, D]."""
    import torch

    B, H, S, D = q.shape
    out = torch.empty_like(q)
    per_head = S * S * 4
    hc = max(1, min(H, max_score_bytes // per_head))
    tri = torch.ones((S, S), dtype=torch.bool, device=q.device).triu(1) if causal else None
    for b in range(B):
        for h0 in range(0, H, hc):
            h1 = min(H, h0 + hc)
            s = torch.matmul(q[b, h0:h1], k[b, h0:h1].transpose(-1, -2)) * scale
            if tri is not None:
                s = s.masked_fill(tri, float("-inf"))
            if mask is not None:
                s = s.masked_fill(~mask[b][None, None, :], float("-inf"))
            p = torch.softmax(s.float(), dim=-1).to(q.dtype)
            out[b, h0:h1] = torch.matmul(p, v[b, h0:h1])
    return out


def run_dense_arm(args, cfg: dict, rank: int, world: int) -> int:
    """Yardstick (not the reference arm): the reference's dense PyTorch attention
    run on this GPU, the path a B200 takes today without this kernel."""
    if rank != 0:
        return 0
    import torch

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    B, H, _ = shard_for(cfg, 1, 0)
    S, D, causal = cfg["S"], cfg["D"], cfg["causal"]
    lengths = valid_lengths(cfg, args.seed)
    flop = flops_for(cfg, B, H, lengths)
    gen = torch.Generator(device=dev).manual_seed(args.seed)
    q, k, v = (torch.randn((B, H, S, D), generator=gen, device=dev).to(cfg_dtype(cfg))
               for _ in range(3))
    mask = None
    if lengths is not None:
        mask = torch.arange(S, device=dev)[None, :] < torch.tensor(lengths, device=dev)[:, None]
    cap = 16 * 2 ** 30
    for _ in range(args.warmup):
        dense_torch_attention(q, k, v, mask, causal, D ** -0.5, cap)
    torch.cuda.synchronize(dev)
    sampler = ClockSampler(0)
    stream = torch.cuda.current_stream(dev)
    with sampler:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            dense_torch_attention(q, k, v, mask, causal, D ** -0.5, cap)
        e1.record(stream)
        torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / args.steps
    line = {
        "impl": "torch-dense", "metric": METRIC, "value": flop / (ms * 1e-3) / 1e12, "unit": UNIT,
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "dtype": dtype_tag(cfg), "data": "synthetic (seeded torch.randn N(0,1))",
        "config": {"workload": args.workload, **{k: cfg[k] for k in ("B", "H", "S", "D", "causal")},
                   "per_gpu_batch_heads": [B, H],
                   "impl_path": "dense torch CUDA ops in _reference_attention's order (cuBLAS GEMMs)"},
        "peak_mem_gb": torch.cuda.max_memory_allocated(dev) / 1e9,
        "clocks": sampler.summary(),
    }
    print(json.dumps(line), flush=True)
    return 0


def run_softmax_arm(args, cfg: dict, rank: int, world: int, local_rank: int, dev, barrier,
                    max_over_ranks) -> int:
    """The row softmax over materialised [B, H, S, S] scores (HBM-bound): value
    = whole-job GB/s of algorithmic bytes (scores read once, probabilities
    written once); inputs rotate over buffers larger than L2."""
    import torch
    import torch.distributed as dist

    from b200_attention import _native
    from b200_attention.fused_attention import read_device_errors
    from b200_attention.softmax import b200_attention_softmax
    from oracle.reference_attention import reference_softmax

    B, H, scaling = shard_for(cfg, world, rank)
    S, D, causal = cfg["S"], cfg["D"], cfg["causal"]
    dtype = cfg_dtype(cfg)
    elem = torch.finfo(dtype).bits // 8
    nbytes = 2.0 * B * H * S * S * elem
    n_sets = max(2, math.ceil(2 * L2_BYTES / (B * H * S * S * elem)))
    gen = torch.Generator(device=dev).manual_seed(args.seed + 1000 * rank)
    scores = [(4 * torch.randn((B, H, S, S), generator=gen, device=dev)).to(dtype)
              for _ in range(n_sets)]
    outs = [torch.empty_like(t) for t in scores]

    def step(i):
        return b200_attention_softmax(scores[i % n_sets], None, D ** -0.5, causal,
                                      out=outs[i % n_sets])

    stream = torch.cuda.current_stream(dev)
    for i in range(max(args.warmup, 3)):
        step(i)
    torch.cuda.synchronize(dev)
    if read_device_errors(dev):
        raise RuntimeError("kernel reported a device error during warm-up")
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    sampler = ClockSampler(local_rank)
    barrier()
    torch.cuda.synchronize(dev)
    launches0 = _native.launch_count()
    with sampler:
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for i in range(args.steps):
            ev[i][0].record(stream)
            step(i)
            ev[i][1].record(stream)
        t1.record(stream)
        torch.cuda.synchronize(dev)
    barrier()
    launches = _native.launch_count() - launches0
    ms_per_step = max_over_ranks(t0.elapsed_time(t1)) / args.steps
    launch_ms = statistics.mean(a.elapsed_time(b) for a, b in ev)
    value = world * nbytes / (ms_per_step * 1e-3) / 1e9

    # end to end: scores up from pinned host memory and probabilities back,
    # every step, through the public operator
    hs = scores[0].cpu().pin_memory()
    ho = torch.empty_like(hs).pin_memory()
    e2e_steps = args.e2e_steps or 3
    d_in, d_out = torch.empty_like(scores[0]), torch.empty_like(scores[0])
    torch.cuda.synchronize(dev)
    barrier()
    t0.record(stream)
    for _ in range(e2e_steps):
        d_in.copy_(hs, non_blocking=True)
        b200_attention_softmax(d_in, None, D ** -0.5, causal, out=d_out)
        ho.copy_(d_out, non_blocking=True)
    t1.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    e2e_ms = max_over_ranks(t0.elapsed_time(t1)) / e2e_steps
    if not torch.equal(ho, outs[0].cpu()):
        raise RuntimeError("end-to-end softmax differs from the device-resident run")

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        torch.set_num_threads(os.cpu_count() or 1)
        heads = max(1, min(H, int(2 ** 31 // (S * S * 12))))
        hs1 = scores[0][:1, :heads].cpu()
        times = []
        while sum(times) < args.cpu_budget or len(times) < 3:
            c0 = time.perf_counter()
            reference_softmax(hs1, None, D ** -0.5, causal)
            times.append(time.perf_counter() - c0)
        med = statistics.median(times)
        sample_bytes = 2.0 * heads * S * S * elem
        cpu = {"value": sample_bytes / med / 1e9, "unit": "GB/s", "cores": torch.get_num_threads(),
               "kind": "port", "ms_per_step_extrapolated": nbytes / (sample_bytes / med) * 1e3,
               "sample": f"{len(times)} reps of oracle.reference_softmax (torch CPU, reference op "
                         f"order) on [1,{heads},{S},{S}]"}
    peaks, peak_src = load_peaks()
    gbs = nbytes / (launch_ms * 1e-3) / 1e9
    roof = {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
            "frac": gbs / peaks["hbm_gbs"], "traffic": None, "algorithmic_bytes": nbytes,
            "avg_launch_ms": launch_ms, "peak_source": f"{peak_src} hbm_gbs",
            "kernel": "softmax_rows_kernel"}
    if world > 1:
        dist.barrier(device_ids=[local_rank])
        dist.destroy_process_group()
    if rank != 0:
        return 0
    line = {
        "metric": "row softmax over materialised attention scores, GB/s", "value": value,
        "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": scaling,
        "vs_baseline": None, "dtype": dtype_tag(cfg), "data": "synthetic (seeded 4 * N(0,1) scores)",
        "config": {"workload": args.workload, "B": B, "H": H, "S": S, "causal": causal,
                   "l2": f"{n_sets} score buffers of {B * H * S * S * elem / 2**20:.0f} MiB (> L2)"},
        "roofline": roof, "cpu_baseline": cpu,
        "e2e": {"value": world * nbytes / (e2e_ms * 1e-3) / 1e9, "unit": "GB/s",
                "h2d_bytes_per_step": hs.numel() * elem, "d2h_bytes_per_step": ho.numel() * elem,
                "ms_per_step": e2e_ms},
        "gpu_launches": launches, "clocks": sampler.summary(),
    }
    print(json.dumps(line), flush=True)
    return 0


def run_context_parallel_arm(args, cfg: dict, rank: int, world: int, local_rank: int, dev,
                             barrier, max_over_ranks) -> int:
    """One long causal sequence sharded over the ranks in zigzag order, K/V
    passed around a ring (NCCL send/recv) while the kernel's partial form
    attends to the chunk at hand.  value = whole-sequence attention TFLOP/s
    (4 B H S^2 D / 2) over the max-over-ranks time; N = 1 runs the same chunk
    pairs on one GPU."""
    import torch
    import torch.distributed as dist

    from b200_attention import _native
    from b200_attention.context_parallel import (b200_partial_attention, ring_attention,
                                                 shard_sequence)
    from b200_attention.fused_attention import b200_fused_attention, read_device_errors

    B, H, S, D = cfg["B"], cfg["H"], cfg["S"], cfg["D"]
    dtype = cfg_dtype(cfg)
    flop = 4.0 * B * H * S * S * D / 2
    gen = torch.Generator(device="cpu").manual_seed(args.seed)
    q, k, v = (torch.randn((B, H, S, D), generator=gen).to(dtype) for _ in range(3))
    shares = [shard_sequence(t, world, rank).to(dev) for t in (q, k, v)]
    scale = D ** -0.5

    def step():
        return ring_attention(*shares, True, scale, b200_partial_attention)[0]

    stream = torch.cuda.current_stream(dev)
    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize(dev)
    if read_device_errors(dev):
        raise RuntimeError("kernel reported a device error during warm-up")
    sampler = ClockSampler(local_rank)
    barrier()
    torch.cuda.synchronize(dev)
    launches0 = _native.launch_count()
    with sampler:
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for _ in range(args.steps):
            out = step()
        t1.record(stream)
        torch.cuda.synchronize(dev)
    barrier()
    launches = _native.launch_count() - launches0
    ms_per_step = max_over_ranks(t0.elapsed_time(t1)) / args.steps
    value = flop / (ms_per_step * 1e-3) / 1e12
    finite = bool(torch.isfinite(out.float()).all())
    single = None
    if world == 1:
        # the same sequence in one plain launch, for the cost of the chunking
        qd, kd, vd = (t.to(dev) for t in (q, k, v))
        b200_fused_attention(qd, kd, vd, None, True)
        torch.cuda.synchronize(dev)
        t0.record(stream)
        for _ in range(3):
            b200_fused_attention(qd, kd, vd, None, True)
        t1.record(stream)
        torch.cuda.synchronize(dev)
        single = flop / (t0.elapsed_time(t1) / 3 * 1e-3) / 1e12
    peaks, peak_src = load_peaks()
    per_gpu = value / world
    if world > 1:
        dist.barrier(device_ids=[local_rank])
        dist.destroy_process_group()
    if rank != 0:
        return 0
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": dtype_tag(cfg),
        "data": "synthetic (seeded torch.randn N(0,1))",
        "config": {"workload": args.workload, "B": B, "H": H, "S": S, "D": D, "causal": True,
                   "parallelism": f"context-parallel x{world}: zigzag sequence shards, K/V ring "
                                  "over NCCL send/recv overlapped with the partial kernel",
                   "chunk_len": S // (2 * world)},
        "roofline": {"bound": "tensor", "achieved": per_gpu, "peak": peaks["bf16_tflops"],
                     "unit": "TFLOP/s", "frac": per_gpu / peaks["bf16_tflops"], "traffic": None,
                     "peak_source": f"{peak_src} bf16_tflops", "per": "GPU (whole-step average)"},
        "single_launch_tflops": single, "gpu_launches": launches, "clocks": sampler.summary(),
        "validation": {"finite": finite},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_model_arm(args, cfg: dict, rank: int, world: int, local_rank: int, dev, barrier,
                  max_over_ranks) -> int:
    """cfg5: forward of the 12-layer decoder whose attention is the sm_100a kernel.

    A step is one forward over this rank's share of the global batch of 8
    sequences (token ids -> embedding -> 12 blocks -> final LayerNorm).  value
    = whole-job decoder TFLOP/s (projections, FFN and causal attention).  The
    attention kernel alone is timed at the same per-rank shape for the
    roofline and the attention share of the forward."""
    import torch
    import torch.distributed as dist

    from b200_attention import _native
    from b200_attention.fused_attention import b200_fused_attention, read_device_errors
    from b200_attention.transformer import Decoder, DecoderConfig, init_normal_

    B, H, scaling = shard_for(cfg, world, rank)
    S, D = cfg["S"], cfg["D"]
    dcfg = DecoderConfig(B, S, cfg["d_model"], H, cfg["ffn"], cfg["layers"], cfg["causal"],
                         vocab_size=cfg["vocab"])
    fused = not args.unfused_epilogues
    model = init_normal_(Decoder(dcfg, fused_epilogues=fused), seed=args.seed)
    model = model.to(device=dev, dtype=torch.bfloat16).eval()
    flop_rank = dcfg.forward_flops()
    tot = torch.tensor([flop_rank], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(tot)
    flop_job = float(tot.item())
    gen = torch.Generator(device="cpu").manual_seed(args.seed + 1000 * rank)
    n_sets = 2
    tokens = [torch.randint(0, cfg["vocab"], (B, S), generator=gen).to(dev) for _ in range(n_sets)]
    stream = torch.cuda.current_stream(dev)

    with torch.inference_mode():
        for i in range(max(args.warmup, 3)):
            model(tokens[i % n_sets])
        torch.cuda.synchronize(dev)
        if read_device_errors(dev):
            raise RuntimeError("kernel reported a device error during warm-up")
        forward = model
        graph = None
        if args.graph:
            # the whole forward captured once (every op, the attention kernel
            # included, launches on the stream without host synchronisation)
            static_tokens = tokens[0].clone()
            graph = torch.cuda.CUDAGraph()
            cap = torch.cuda.Stream(dev)
            cap.wait_stream(stream)
            with torch.cuda.stream(cap):
                model(static_tokens)
                cap.synchronize()
                c0 = _native.launch_count()
                with torch.cuda.graph(graph, stream=cap):
                    static_out = model(static_tokens)
                graph_launches = _native.launch_count() - c0
            stream.wait_stream(cap)

            def forward(tok):
                static_tokens.copy_(tok, non_blocking=True)
                graph.replay()
                return static_out
        sampler = ClockSampler(local_rank)
        barrier()
        torch.cuda.synchronize(dev)
        launches0 = _native.launch_count()
        with sampler:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for i in range(args.steps):
                out = forward(tokens[i % n_sets])
            e1.record(stream)
            torch.cuda.synchronize(dev)
        barrier()
        # this package's kernel launches inside the timed region (a graph's
        # launches were counted once, at capture, and replay once per step)
        launches = (graph_launches * args.steps if graph is not None
                    else _native.launch_count() - launches0)
        ms_per_step = max_over_ranks(e0.elapsed_time(e1)) / args.steps
        value = flop_job / (ms_per_step * 1e-3) / 1e12
        finite = bool(torch.isfinite(out.float()).all())

        # the attention kernel alone at this rank's shape (per-launch events)
        g2 = torch.Generator(device=dev).manual_seed(args.seed)
        q, k, v = (torch.randn((B, H, S, D), generator=g2, device=dev).to(torch.bfloat16)
                   for _ in range(3))
        for _ in range(3):
            b200_fused_attention(q, k, v, None, True)
        torch.cuda.synchronize(dev)
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(20)]
        for a, b in ev:
            a.record(stream)
            b200_fused_attention(q, k, v, None, True)
            b.record(stream)
        torch.cuda.synchronize(dev)
        attn_ms = statistics.mean(a.elapsed_time(b) for a, b in ev)
        attn_flop = 4.0 * B * H * S * S * D / 2
        errors = read_device_errors(dev)

        # end to end: token ids from pinned host memory, output back to the host,
        # every step.  Steps are pipelined the way a server streams batches: the
        # forward of step i+1 runs while step i's output is copied to the host on
        # a copy stream (two device staging buffers, two pinned host buffers).
        htoks = [t.cpu().pin_memory() for t in tokens]
        houts = [torch.empty((B, S, cfg["d_model"]), dtype=torch.bfloat16).pin_memory()
                 for _ in range(2)]
        stage = [torch.empty((B, S, cfg["d_model"]), dtype=torch.bfloat16, device=dev)
                 for _ in range(2)]
        d2h_stream = torch.cuda.Stream(dev)
        copied = [torch.cuda.Event() for _ in range(2)]

        def e2e_step(i):
            j = i % 2
            stream.wait_event(copied[j])  # step i-2's download has left stage[j]
            out_i = forward(htoks[i % n_sets].to(dev, non_blocking=True))
            stage[j].copy_(out_i, non_blocking=True)
            d2h_stream.wait_stream(stream)
            with torch.cuda.stream(d2h_stream):
                houts[j].copy_(stage[j], non_blocking=True)
                copied[j].record(d2h_stream)

        for i in range(2):
            e2e_step(i)
        torch.cuda.synchronize(dev)
        barrier()
        e2e_steps = args.e2e_steps or max(3, min(args.steps, 10))
        e0.record(stream)
        for i in range(e2e_steps):
            e2e_step(i)
        stream.wait_stream(d2h_stream)
        e1.record(stream)
        torch.cuda.synchronize(dev)
        barrier()
        hout = houts[(e2e_steps - 1) % 2]
        # the last download equals a fresh forward of the same tokens (every
        # kernel on the path is deterministic)
        e2e_exact = bool(torch.equal(hout, forward(tokens[(e2e_steps - 1) % n_sets]).cpu()))
        e2e_ms = max_over_ranks(e0.elapsed_time(e1)) / e2e_steps

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = CpuReference(cfg, args.seed).measure(args.cpu_budget, min_reps=3)
        cpu["sample"] += " (the decoder's attention core; no CPU decoder is timed)"
    peaks, peak_src = load_peaks()
    traffic, traffic_src = None, None
    if world == 1:  # captured at the N = 1 per-layer shape
        traffic, traffic_src = stored_traffic("attn_fwd_sm100_cfg5_traffic.json")
    roof = roofline(attn_flop, algorithmic_bytes(cfg, B, H, None), attn_ms, peaks, peak_src,
                    traffic, traffic_src)
    roof["kernel"] = "attn_fwd_sm100_kernel at the per-rank attention shape of one layer"
    if world > 1:
        dist.barrier(device_ids=[local_rank])
        dist.destroy_process_group()
    if rank != 0:
        return 0
    attn_tflops = attn_flop / (attn_ms * 1e-3) / 1e12
    line = {
        "metric": METRIC, "value": value, "unit": "TFLOP/s (decoder forward)", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
        "higher_is_better": True, "scaling": scaling, "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (uniform random token ids, random-init weights N(0, 0.02))",
        "config": {"workload": "cfg5", "layers": cfg["layers"], "d_model": cfg["d_model"],
                   "heads": H, "head_dim": D, "ffn": cfg["ffn"], "vocab": cfg["vocab"],
                   "global_batch": cfg["B"], "per_rank_batch": B, "seq_len": S, "causal": True,
                   "parallelism": f"data-parallel batch split x{world}, no data-path collective",
                   "launch": "CUDA graph of the whole forward" if graph is not None else "eager",
                   "epilogues": ("fused linear kernel: out_proj + residual, ffn_in + GELU "
                                 "(QKV and ffn_out on cuBLAS); LayerNorm kernel with the "
                                 "blocks' closing residual add folded in") if fused else
                                "cuBLAS linear layers + separate GELU / add passes; torch LayerNorm",
                   "l2": f"{n_sets} token sets; each forward streams ~0.4 GB of weights and activations (> L2)",
                   "flop_per_step_job": flop_job},
        "attention": {"tflops": attn_tflops, "ms_per_layer": attn_ms,
                      "share_of_forward": cfg["layers"] * attn_ms / ms_per_step},
        "roofline": roof,
        "cpu_baseline": cpu,
        "e2e": {"value": flop_rank / (e2e_ms * 1e-3) / 1e12 * world, "unit": "TFLOP/s (decoder forward)",
                "h2d_bytes_per_step": htoks[0].numel() * htoks[0].element_size(),
                "d2h_bytes_per_step": hout.numel() * hout.element_size(), "ms_per_step": e2e_ms,
                "pipelining": "step i+1's forward overlaps step i's download (copy stream)"},
        "gpu_launches": launches,
        "clocks": sampler.summary(),
        "validation": {"finite": finite, "device_errors": errors, "e2e_bit_exact": e2e_exact},
    }
    print(json.dumps(line), flush=True)
    return 0


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--workload", default="cfg4", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="b200", choices=["b200", "reference", "torch-dense"])
    ap.add_argument("--e2e-steps", type=int, default=None)
    ap.add_argument("--cpu-budget", type=float, default=10.0, help="seconds of CPU baseline work")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--seed", type=int, default=1234)
    ap.add_argument("--graph", action="store_true",
                    help="replay the timed steps from a CUDA graph (launch-bound workloads)")
    ap.add_argument("--heads", type=int, default=None,
                    help="override the workload's head count (smaller cases for profiler "
                         "captures; the line's config records it)")
    ap.add_argument("--unfused-epilogues", action="store_true",
                    help="cfg5: run the block's linear layers on cuBLAS with separate GELU/add "
                         "passes (the yardstick for the fused linear kernel)")
    args = ap.parse_args(argv)
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")

    cfg = dict(WORKLOADS[args.workload])
    if args.heads is not None:
        cfg["H"] = args.heads
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        return run_reference_arm(args, cfg, rank, world)
    if args.impl == "torch-dense":
        return run_dense_arm(args, cfg, rank, world)

    import torch
    import torch.distributed as dist

    from b200_attention import _native
    from b200_attention.fused_attention import b200_fused_attention, read_device_errors

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    if args.workload == "cfg5":
        return run_model_arm(args, cfg, rank, world, local_rank, dev, barrier, max_over_ranks)
    if cfg.get("kind") == "softmax":
        return run_softmax_arm(args, cfg, rank, world, local_rank, dev, barrier, max_over_ranks)
    if cfg.get("kind") == "context_parallel":
        return run_context_parallel_arm(args, cfg, rank, world, local_rank, dev, barrier,
                                        max_over_ranks)

    B, H, scaling = shard_for(cfg, world, rank)
    S, D, causal = cfg["S"], cfg["D"], cfg["causal"]
    lengths = valid_lengths(cfg, args.seed)
    flop_rank = flops_for(cfg, B, H, lengths)
    tot = torch.tensor([flop_rank], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(tot)
    flop_job = float(tot.item())

    # ---- inputs: rotate over enough buffers that their total exceeds L2
    bytes_per_set = 4 * B * H * S * D * 2
    n_sets = max(2, math.ceil(2 * L2_BYTES / bytes_per_set))
    gen = torch.Generator(device=dev).manual_seed(args.seed + 1000 * rank)
    sets = []
    for _ in range(n_sets):
        q, k, v = (torch.randn((B, H, S, D), generator=gen, device=dev, dtype=torch.float32)
                   .to(cfg_dtype(cfg)) for _ in range(3))
        sets.append((q, k, v))
    mask = None
    if lengths is not None:
        mask = (torch.arange(S, device=dev)[None, :] <
                torch.tensor(lengths, device=dev)[:, None])
    outs = [torch.empty((B, S, H, D), device=dev, dtype=cfg_dtype(cfg)) for _ in range(n_sets)]
    zero_q = mask is not None

    def step(i):
        q, k, v = sets[i % n_sets]
        return b200_fused_attention(q, k, v, mask, causal, output_bshd=True,
                                    zero_masked_queries=zero_q, out=outs[i % n_sets])

    stream = torch.cuda.current_stream(dev)
    # W warm-up steps, continued until ~0.5 s of work so clocks leave idle
    t_w = time.perf_counter()
    i = 0
    while i < args.warmup or time.perf_counter() - t_w < 0.5:
        step(i)
        i += 1
        if i % 8 == 0:
            torch.cuda.synchronize(dev)
    torch.cuda.synchronize(dev)
    if read_device_errors(dev):
        raise RuntimeError("kernel reported a device error during warm-up")

    # ---- device-resident timed region.  Per-launch durations (roofline.achieved)
    # come from event pairs around every SAMPLE-th launch of the timed region:
    # a torch event record costs ~5 us of host time, and a pair on every step
    # would make short launches (cfg1: 11 us) host-bound on the bench itself.
    sample = 8
    sampled = list(range(0, args.steps, sample))
    ev = {i: (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for i in sampled}
    graph = None
    if args.graph:
        # the K steps captured once and replayed: no host work inside the timed
        # region (for launch-bound workloads such as cfg1)
        graph = torch.cuda.CUDAGraph()
        cap = torch.cuda.Stream(dev)
        cap.wait_stream(stream)
        with torch.cuda.stream(cap):
            step(0)
            cap.synchronize()
            c0 = _native.launch_count()
            with torch.cuda.graph(graph, stream=cap):
                for i in range(args.steps):
                    step(i)
            graph_launches = _native.launch_count() - c0
        stream.wait_stream(cap)
        graph.replay()
        torch.cuda.synchronize(dev)
    sampler = ClockSampler(local_rank)
    barrier()
    torch.cuda.synchronize(dev)
    launches0 = _native.launch_count()
    with sampler:
        t_start = torch.cuda.Event(enable_timing=True)
        t_end = torch.cuda.Event(enable_timing=True)
        t_start.record(stream)
        if graph is not None:
            graph.replay()
        else:
            for i in range(args.steps):
                pair = ev.get(i)
                if pair is not None:
                    pair[0].record(stream)
                    step(i)
                    pair[1].record(stream)
                else:
                    step(i)
        t_end.record(stream)
        torch.cuda.synchronize(dev)
    barrier()
    # launches the library issued inside the timed region (a graph's launches
    # were counted once, at capture)
    launches = graph_launches if graph is not None else _native.launch_count() - launches0
    elapsed_ms = max_over_ranks(t_start.elapsed_time(t_end))
    if graph is not None:
        avg_launch_ms = t_start.elapsed_time(t_end) / args.steps  # back-to-back launches
    else:
        avg_launch_ms = statistics.mean(a.elapsed_time(b) for a, b in ev.values())
    errors = read_device_errors(dev)
    ms_per_step = elapsed_ms / args.steps
    value = flop_job / (ms_per_step * 1e-3) / 1e12

    # ---- validation gather (outside the timed region): finiteness and a checksum per rank
    o = outs[(args.steps - 1) % n_sets].float()
    finite = torch.isfinite(o).all()
    check = torch.stack([o.abs().sum(dtype=torch.float64), finite.double(),
                         torch.tensor(float(errors), device=dev, dtype=torch.float64)])
    gathered = [torch.zeros_like(check) for _ in range(world)]
    if world > 1:
        dist.all_gather(gathered, check)
    else:
        gathered = [check]
    validation = {"finite_all_ranks": all(bool(g[1].item()) for g in gathered),
                  "device_errors": int(sum(g[2].item() for g in gathered)),
                  "checksums": [round(float(g[0].item()), 3) for g in gathered]}

    # ---- end to end through the public operator with pinned host buffers.
    # Every step copies its Q, K, V (and mask) host->device, runs the operator
    # and copies the output device->host.  Steps are pipelined the way a
    # server streams batches: uploads on one stream, the operator on the
    # compute stream, downloads on a third, two device buffer sets, so the
    # two PCIe directions and the kernel overlap across steps.
    e2e_steps = args.e2e_steps or max(3, min(args.steps, 20))
    hq, hk, hv = (t.cpu().pin_memory() for t in sets[0])
    hmask = mask.cpu().pin_memory() if mask is not None else None
    houts = [torch.empty((B, S, H, D), dtype=cfg_dtype(cfg)).pin_memory() for _ in range(2)]
    h2d = 3 * hq.numel() * hq.element_size() + (hmask.numel() if hmask is not None else 0)
    d2h = houts[0].numel() * houts[0].element_size()
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    dev_in = [[torch.empty_like(t, device=dev) for t in (hq, hk, hv)] for _ in range(2)]
    dev_mask = [torch.empty_like(hmask, device=dev) if hmask is not None else None for _ in range(2)]
    dev_out = [torch.empty((B, S, H, D), device=dev, dtype=cfg_dtype(cfg)) for _ in range(2)]
    ev = {name: [torch.cuda.Event() for _ in range(2)] for name in ("in", "comp", "out")}
    for name in ev:
        for e in ev[name]:
            e.record(stream)

    def e2e_step(i):
        b = i % 2
        with torch.cuda.stream(s_in):
            s_in.wait_event(ev["comp"][b])  # buffer set b no longer read by the operator
            for dst, src in zip(dev_in[b], (hq, hk, hv)):
                dst.copy_(src, non_blocking=True)
            if hmask is not None:
                dev_mask[b].copy_(hmask, non_blocking=True)
            ev["in"][b].record(s_in)
        stream.wait_event(ev["in"][b])
        stream.wait_event(ev["out"][b])  # previous download of output b finished
        b200_fused_attention(*dev_in[b], dev_mask[b], causal, output_bshd=True,
                             zero_masked_queries=zero_q, out=dev_out[b])
        ev["comp"][b].record(stream)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev["comp"][b])
            houts[b].copy_(dev_out[b], non_blocking=True)
            ev["out"][b].record(s_out)

    for i in range(3):
        e2e_step(i)
    torch.cuda.synchronize(dev)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    s_in.wait_stream(stream)
    for i in range(e2e_steps):
        e2e_step(i)
    stream.wait_stream(s_out)
    stream.wait_stream(s_in)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1)) / e2e_steps
    e2e_value = flop_job / (e2e_ms * 1e-3) / 1e12
    if not torch.equal(houts[(e2e_steps - 1) % 2], outs[0].cpu()):
        raise RuntimeError("end-to-end output differs from the device-resident run on the same inputs")

    # ---- CPU baseline (rank 0, N = 1 only)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = CpuReference(cfg, args.seed).measure(args.cpu_budget, min_reps=3, full_flop=flop_job)

    peaks, peak_src = load_peaks()
    peak = peaks["bf16_tflops"]
    # captured for the whole N = 1 launch; a head-sharded rank processes
    # H / cfg["H"] of the heads, and the traffic scales with them
    traffic, traffic_src = stored_traffic(f"attn_fwd_sm100_{args.workload}_traffic.json",
                                          H / cfg["H"])
    roof = roofline(flop_rank, algorithmic_bytes(cfg, B, H, lengths), avg_launch_ms, peaks,
                    peak_src, traffic, traffic_src)

    vs_baseline = None
    if "published_ms" in cfg:
        # the reference's own number for this shape, on other hardware
        vs_baseline = value / (flops_for(cfg, cfg["B"], cfg["H"], None) / (cfg["published_ms"] * 1e-3) / 1e12)
    if world > 1:
        dist.barrier(device_ids=[local_rank])
        dist.destroy_process_group()
    if rank != 0:
        return 0
    line = {
        "metric": METRIC,
        "value": value,
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_per_step,
        "higher_is_better": True,
        "scaling": scaling,
        "vs_baseline": vs_baseline,
        "dtype": dtype_tag(cfg),
        "data": "synthetic (seeded torch.randn N(0,1), no dataset)",
        "config": {
            "workload": args.workload, "B": cfg["B"], "H": cfg["H"], "S": S, "D": D,
            "causal": causal, "key_padding": lengths is not None,
            "per_rank_batch_heads": [B, H],
            "parallelism": f"{'bxh' if scaling == 'weak' else 'heads'}-shard x{world}, no data-path collective",
            "l2": f"inputs rotated over {n_sets} buffer sets of {bytes_per_set / 2**20:.0f} MiB (> L2)",
            "launch": "CUDA graph of the timed steps" if graph is not None else "eager, one operator call per step",
            "launch_timing": ("graph replay time / steps" if graph is not None else
                              f"CUDA events around every {sample}th launch of the timed region "
                              f"({len(sampled)} launches)"),
            "flop_per_step_job": flop_job,
            "valid_lengths": lengths,
            **({"published_baseline": f"{cfg['published_hw']}: {cfg['published_ms']} ms per call "
                                      "(vs_baseline compares across hardware)"}
               if "published_ms" in cfg else {}),
        },
        "pct_of_bf16_peak": 100.0 * value / (peak * world),
        "roofline": roof,
        "cpu_baseline": cpu,
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "ms_per_step": e2e_ms,
                "mode": "steps pipelined: uploads, operator and downloads on three streams"},
        "gpu_launches": launches,
        "clocks": sampler.summary(),
        "validation": validation,
    }
    if cpu:
        line["speedup_vs_cpu_e2e"] = e2e_value / cpu["value"]
    print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
