"""Context-parallel attention on the GPU: the kernel's partial form
(``b200_attn_fwd_partial``) over the zigzag chunk pairs of N ranks, run in
one process on one GPU (every virtual rank's pairs in turn, no exchange), and
on two GPUs with the NCCL ring when the box has them.  The assembled output
must match the oracle on the whole sequence within the stated tolerance
(max-abs <= 2e-2, mean-abs <= 2e-3); the per-row log-sum-exp must match the
exact fp32 log-sum-exp of the scaled scores within 2e-2 (the exact-rounding
rows round the scores to the input dtype first)."""

import os
import socket

import pytest
import torch

from b200_attention import read_device_errors
from b200_attention.context_parallel import (b200_partial_attention, chunk_pairs, ring_attention,
                                             shard_sequence, unshard_sequence)
from oracle.reference_attention import reference_attention
from parity import assert_close, seeded_qkv

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def _exact_lse(q, k, causal, scale):
    s = torch.matmul(q.float(), k.float().transpose(-1, -2)) * scale
    if causal:
        S = s.shape[-1]
        s = s.masked_fill(torch.ones(S, S, dtype=torch.bool).triu(1), float("-inf"))
    return torch.logsumexp(s, -1)


def _emulated_ranks(q, k, v, world, causal, scale):
    """Every virtual rank's chunk pairs on this GPU, as the ring would run them."""
    outs, lses = [], []
    shares = [[shard_sequence(t, world, r).to(DEV) for t in (q, k, v)] for r in range(world)]
    L = q.shape[2] // (2 * world)
    for r in range(world):
        qr = shares[r][0]
        out = torch.empty_like(qr)
        lse = torch.empty(qr.shape[:3], device=DEV, dtype=torch.float32)
        started = [False, False]
        for step in range(world):
            src = (r - step) % world
            ks, vs = shares[src][1], shares[src][2]
            for qi, ki, diag in chunk_pairs(world, r, src, causal):
                qsl, ksl = slice(qi * L, (qi + 1) * L), slice(ki * L, (ki + 1) * L)
                b200_partial_attention(qr[:, :, qsl], ks[:, :, ksl], vs[:, :, ksl], diag, scale,
                                       out[:, :, qsl], lse[:, :, qsl], started[qi])
                started[qi] = True
        outs.append(out.cpu())
        lses.append(lse.cpu())
    torch.cuda.synchronize()
    assert read_device_errors(DEV) == 0
    return unshard_sequence(outs), unshard_sequence(lses)


@pytest.mark.parametrize("world", [1, 2, 4])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("causal", [True, False])
def test_emulated_ring_matches_whole_sequence_attention(world, dtype, causal):
    D = 64 if dtype == torch.float32 else 128
    B, H, S = 1, 2, 2 * world * 256 + (0 if world > 1 else 512)
    q, k, v = seeded_qkv((B, H, S, D), dtype, 5 + world)
    scale = D ** -0.5
    out, lse = _emulated_ranks(q, k, v, world, causal, scale)
    ref = reference_attention(q, k, v, None, causal, scale)
    assert_close(out, ref, f"cp world={world} {dtype} causal={causal}")
    d = (lse - _exact_lse(q, k, causal, scale)).abs()
    assert float(d.max()) <= 2e-2, float(d.max())


def test_partial_chunk_lengths_not_multiple_of_tile():
    """Chunks of 200 rows (partial 128-row tiles) over 2 virtual ranks."""
    q, k, v = seeded_qkv((2, 2, 800, 64), torch.bfloat16, 17)
    out, _ = _emulated_ranks(q, k, v, 2, True, 0.125)
    assert_close(out, reference_attention(q, k, v, None, True, 0.125), "cp ragged chunks")


def test_partial_form_rejects_masks():
    from b200_attention import _native
    q = torch.zeros((1, 1, 128, 64), device=DEV, dtype=torch.bfloat16)
    lse = torch.zeros((1, 1, 128), device=DEV)
    with pytest.raises(ValueError):
        b200_partial_attention(q, q, q, True, 0.125, torch.empty_like(q), lse[:, :, :64], False)
    assert _native.ERR_UNSUPPORTED == 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_worker(rank, world, port, results):
    import datetime

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        q, k, v = seeded_qkv((1, 4, 4 * world * 256, 128), torch.bfloat16, 23)
        shares = [shard_sequence(t, world, rank).to(dev) for t in (q, k, v)]
        out, _ = ring_attention(*shares, True, 128 ** -0.5, b200_partial_attention)
        gathered = [torch.empty_like(out) for _ in range(world)]
        dist.all_gather(gathered, out)
        if rank == 0:
            full = unshard_sequence([g.cpu() for g in gathered])
            ref = reference_attention(q, k, v, None, True, 128 ** -0.5)
            d = (full.float() - ref.float()).abs()
            results.put((float(d.max()), float(d.mean())))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_nccl_ring_on_two_gpus_matches_whole_sequence_attention():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_nccl_worker, args=(r, 2, port, results)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    max_abs, mean_abs = results.get(timeout=10)
    assert max_abs <= 2e-2 and mean_abs <= 2e-3, (max_abs, mean_abs)
