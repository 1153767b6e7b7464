"""Context-parallel attention on CPU: the zigzag sharding, the chunk-pair
schedule and the ring exchange (gloo, world size 2 and 3) against exact
attention of the whole sequence.  The per-pair compute is a CPU stand-in
(``cp_reference.cpu_partial``); the GPU tests run the kernel's partial form."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from b200_attention.context_parallel import (chunk_pairs, ring_attention, shard_sequence,
                                             unshard_sequence, zigzag_chunk_ids)
from cp_reference import cpu_partial


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_zigzag_shards_round_trip_and_balance(world):
    x = torch.arange(2 * world * 3 * 5).view(1, 1, 2 * world * 3, 5)
    parts = [shard_sequence(x, world, r) for r in range(world)]
    assert torch.equal(unshard_sequence(parts), x)
    ids = sorted(c for r in range(world) for c in zigzag_chunk_ids(world, r))
    assert ids == list(range(2 * world))
    for r in range(world):
        causal = sum(len(chunk_pairs(world, r, s, True)) for s in range(world))
        full = sum(len(chunk_pairs(world, r, s, False)) for s in range(world))
        assert causal == 2 * world + 1 and full == 4 * world


@pytest.mark.parametrize("world", [1, 2, 4])
def test_chunk_pairs_cover_exactly_the_visible_blocks(world):
    """Across ranks and sources, every (query chunk, key chunk) block with a
    visible key appears once, the diagonal causal, the rest full."""
    seen = {}
    for r in range(world):
        q_ids = zigzag_chunk_ids(world, r)
        for s in range(world):
            k_ids = zigzag_chunk_ids(world, s)
            for qi, ki, diag in chunk_pairs(world, r, s, True):
                key = (q_ids[qi], k_ids[ki])
                assert key not in seen
                seen[key] = diag
    n = 2 * world
    assert set(seen) == {(a, b) for a in range(n) for b in range(n) if b <= a}
    assert all(diag == (a == b) for (a, b), diag in seen.items())


def _exact(q, k, v, causal, scale):
    s = torch.matmul(q.float(), k.float().transpose(-1, -2)) * scale
    if causal:
        S = s.shape[-1]
        s = s.masked_fill(torch.ones(S, S, dtype=torch.bool).triu(1), float("-inf"))
    return torch.matmul(torch.softmax(s, -1), v.float()), torch.logsumexp(s, -1)


def test_single_rank_ring_equals_exact_attention():
    gen = torch.Generator().manual_seed(3)
    q, k, v = (torch.randn(2, 3, 64, 16, generator=gen) for _ in range(3))
    out, lse = ring_attention(shard_sequence(q, 1, 0), shard_sequence(k, 1, 0),
                              shard_sequence(v, 1, 0), True, 0.25, cpu_partial)
    ref, ref_lse = _exact(q, k, v, True, 0.25)
    assert torch.allclose(unshard_sequence([out]), ref, atol=1e-5)
    assert torch.allclose(unshard_sequence([lse]), ref_lse, atol=1e-5)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _ring_worker(rank, world, port, causal, results):
    import datetime

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=30))
    try:
        gen = torch.Generator().manual_seed(11)
        q, k, v = (torch.randn(1, 2, 4 * world * 6, 8, generator=gen) for _ in range(3))
        shares = [shard_sequence(t, world, rank) for t in (q, k, v)]
        out, lse = ring_attention(*shares, causal, 8 ** -0.5, cpu_partial)
        gathered = [torch.empty_like(out) for _ in range(world)]
        dist.all_gather(gathered, out)
        lses = [torch.empty_like(lse) for _ in range(world)]
        dist.all_gather(lses, lse)
        if rank == 0:
            ref, ref_lse = _exact(q, k, v, causal, 8 ** -0.5)
            results.put((float((unshard_sequence(gathered) - ref).abs().max()),
                         float((unshard_sequence(lses) - ref_lse).abs().max())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,causal", [(2, True), (2, False), (3, True)])
def test_ring_exchange_on_gloo_ranks_equals_exact_attention(world, causal):
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ring_worker, args=(r, world, port, causal, results))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    err, lse_err = results.get(timeout=10)
    assert err < 1e-5 and lse_err < 1e-5, (err, lse_err)
