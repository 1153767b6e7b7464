"""Multi-rank host logic on CPU: gloo world_size 2 (no GPU).

Each rank computes its contiguous head range with the CPU oracle standing in
for the kernel, then ``gather_heads`` reassembles [B, H, S, D]; rank 0 checks
it against the unsharded oracle.  A second test makes one rank leave before
the validation gather and checks that the survivor's collective ends with an
error inside the short process-group timeout instead of waiting forever.
"""

import datetime
import os
import socket
import traceback

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from b200_attention.sharding import balance_batches, gather_heads, head_ranges, head_shard


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_head_ranges_and_balance():
    assert head_ranges(32, 8) == [(4 * r, 4 * r + 4) for r in range(8)]
    assert head_ranges(5, 2) == [(0, 2), (2, 5)]
    assert sum(hi - lo for lo, hi in head_ranges(17, 4)) == 17
    owners = balance_batches([16, 1, 9, 4, 9], 2)
    assert sorted(sum(owners, [])) == [0, 1, 2, 3, 4]
    loads = [sum([16, 1, 9, 4, 9][b] for b in o) for o in owners]
    assert max(loads) - min(loads) <= 4
    with pytest.raises(ValueError):
        head_ranges(4, 0)


def _worker(rank, world, port, mode, results):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world,
                               timeout=datetime.timedelta(seconds=5))
        import sys
        from pathlib import Path
        root = Path(__file__).resolve().parents[1]
        sys.path[:0] = [str(root / "techjam-kernel_b200"), str(root)]
        from oracle.reference_attention import reference_attention

        gen = torch.Generator().manual_seed(99)
        B, H, S, D = 2, 5, 96, 64
        q, k, v = (torch.randn((B, H, S, D), generator=gen).bfloat16() for _ in range(3))
        if mode == "gather":
            local = reference_attention(head_shard(q, rank, world), head_shard(k, rank, world),
                                        head_shard(v, rank, world), None, True, D ** -0.5)
            full = gather_heads(local, H, world)
            if rank == 0:
                ref = reference_attention(q, k, v, None, True, D ** -0.5)
                results[rank] = bool(torch.equal(full, ref))
            else:
                results[rank] = True
            dist.destroy_process_group()
        else:  # rank 1 leaves before the collective
            if rank == 1:
                results[rank] = True
                return
            try:
                gather_heads(torch.zeros(B, 3, S, D), H, world)
                results[rank] = "no error"
            except Exception as exc:  # timeout or connection closed
                results[rank] = f"error: {type(exc).__name__}"
    except Exception:
        results[rank] = traceback.format_exc()


def _spawn(mode):
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, results)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
            pytest.fail("rank did not finish")
    return dict(results)


def test_gloo_head_shard_gather_equals_unsharded():
    res = _spawn("gather")
    assert res == {0: True, 1: True}, res


def test_gloo_missing_rank_ends_with_error():
    res = _spawn("leave")
    assert res[1] is True
    assert isinstance(res[0], str) and res[0].startswith("error"), res
