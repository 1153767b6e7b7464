"""Context-parallel attention: one sequence sharded over several GPUs.

The reference runs every sequence on one device; a sequence whose attention
does not fit one GPU (or whose latency should drop with more GPUs) is split
here along the sequence into 2N chunks of equal length for N ranks, in the
zigzag order that balances causal work: rank r holds chunks r and 2N-1-r of
Q, K and V.  The K/V chunks travel around a ring of ranks (NCCL send/recv
over NVLink, into a local staging buffer, overlapped with the attention of
the chunk already here).  Each (query chunk, key chunk) pair the causal mask
leaves visible is one call of the kernel's partial form
(``b200_attn_fwd_partial``), which merges the chunk's result into the output
and its per-row log-sum-exp in its epilogue.  Per rank: 2N + 1 chunk pairs
for every rank (causal) or 4N (non-causal).

Test hooks: ``ring_attention`` takes the per-pair compute as an argument, so
the exchange and the schedule run with a CPU stand-in on gloo ranks; the
product path passes ``b200_partial_attention``.
"""

from __future__ import annotations

import ctypes
from typing import Callable, Optional

import torch

from . import _native
from .fused_attention import SUPPORTED_DTYPES, device_error_word, make_params, raise_for_code


def zigzag_chunk_ids(world: int, rank: int) -> tuple[int, int]:
    """The two sequence chunks (of 2 * world) that ``rank`` holds."""
    return rank, 2 * world - 1 - rank


def shard_sequence(x: torch.Tensor, world: int, rank: int, dim: int = 2) -> torch.Tensor:
    """``rank``'s zigzag share of ``x`` along ``dim``: chunks r and 2N-1-r
    concatenated (the sequence length must divide into 2N chunks)."""
    S = x.shape[dim]
    if S % (2 * world):
        raise ValueError(f"sequence length {S} does not split into {2 * world} equal chunks")
    chunks = x.chunk(2 * world, dim=dim)
    a, b = zigzag_chunk_ids(world, rank)
    return torch.cat([chunks[a], chunks[b]], dim=dim)


def unshard_sequence(parts: list[torch.Tensor], dim: int = 2) -> torch.Tensor:
    """Inverse of ``shard_sequence`` given every rank's share (rank order)."""
    world = len(parts)
    chunks: list[Optional[torch.Tensor]] = [None] * (2 * world)
    for r, part in enumerate(parts):
        lo, hi = part.chunk(2, dim=dim)
        a, b = zigzag_chunk_ids(world, r)
        chunks[a], chunks[b] = lo, hi
    return torch.cat(chunks, dim=dim)


def chunk_pairs(world: int, rank: int, source: int, causal: bool) -> list[tuple[int, int, bool]]:
    """The (local query chunk, source key chunk, causal) products ``rank`` runs
    on the K/V of ``source``: a key chunk wholly before the query chunk is
    full attention, the same chunk is the causal diagonal, a later one is
    skipped."""
    q_ids = zigzag_chunk_ids(world, rank)
    k_ids = zigzag_chunk_ids(world, source)
    pairs = []
    for qi, qc in enumerate(q_ids):
        for ki, kc in enumerate(k_ids):
            if not causal:
                pairs.append((qi, ki, False))
            elif kc < qc:
                pairs.append((qi, ki, False))
            elif kc == qc:
                pairs.append((qi, ki, True))
    return pairs


_comm_streams: dict = {}


def _comm_stream(device: torch.device) -> "torch.cuda.Stream":
    """The side stream the ring's K/V exchange runs on (one per device)."""
    stream = _comm_streams.get(device)
    if stream is None:
        stream = _comm_streams[device] = torch.cuda.Stream(device)
    return stream


PartialFn = Callable[[torch.Tensor, torch.Tensor, torch.Tensor, bool, float, torch.Tensor,
                      torch.Tensor, bool], None]


def ring_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool, scale: float,
                   partial: PartialFn, group=None) -> tuple[torch.Tensor, torch.Tensor]:
    """Attention of this rank's zigzag share ``q, k, v`` ([B, H, 2L, D], chunks
    r and 2N-1-r of the sequence) against the whole sequence.  Returns the
    output share [B, H, 2L, D] and its per-row log-sum-exp [B, H, 2L] (fp32).
    ``partial(q_chunk, k_chunk, v_chunk, causal, scale, out_chunk, lse_chunk,
    accumulate)`` computes one chunk pair in place."""
    import torch.distributed as dist

    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    B, H, S2, D = q.shape
    if k.shape != q.shape or v.shape != q.shape or S2 % 2:
        raise ValueError("q, k and v must be [B, H, 2L, D] zigzag shares of one shape")
    L = S2 // 2
    out = torch.empty_like(q)
    lse = torch.empty((B, H, S2), device=q.device, dtype=torch.float32)
    started = [False, False]
    kv = torch.stack([k, v]).contiguous()  # [2, B, H, 2L, D]: this rank's K/V share
    recv = torch.empty_like(kv) if world > 1 else None
    comm = _comm_stream(q.device) if (world > 1 and q.is_cuda) else None
    compute = torch.cuda.current_stream(q.device) if q.is_cuda else None
    for step in range(world):
        source = (rank - step) % world
        pending = None
        if world > 1 and step + 1 < world:
            # send what is here to the next rank, receive the previous rank's
            nxt, prv = (rank + 1) % world, (rank - 1) % world
            if comm is not None:
                comm.wait_stream(compute)
                with torch.cuda.stream(comm):
                    ops = [dist.P2POp(dist.isend, kv, nxt, group), dist.P2POp(dist.irecv, recv, prv, group)]
                    pending = dist.batch_isend_irecv(ops)
            else:
                ops = [dist.P2POp(dist.isend, kv, nxt, group), dist.P2POp(dist.irecv, recv, prv, group)]
                pending = dist.batch_isend_irecv(ops)
        for qi, ki, diag in chunk_pairs(world, rank, source, causal):
            qs = slice(qi * L, (qi + 1) * L)
            ks = slice(ki * L, (ki + 1) * L)
            partial(q[:, :, qs], kv[0][:, :, ks], kv[1][:, :, ks], diag, scale, out[:, :, qs],
                    lse[:, :, qs], started[qi])
            started[qi] = True
        if pending is not None:
            for work in pending:
                work.wait()
            if comm is not None:
                compute.wait_stream(comm)
            kv, recv = recv, kv
    return out, lse


def b200_partial_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool,
                           scale: float, out: torch.Tensor, lse: torch.Tensor,
                           accumulate: bool) -> None:
    """One chunk pair on the sm_100a kernel's partial form (in place on
    ``out`` [B, H, L, D] and ``lse`` [B, H, L] fp32)."""
    if q.dtype not in SUPPORTED_DTYPES or not q.is_cuda:
        raise ValueError("b200_partial_attention takes CUDA bfloat16, float16 or float32 tensors")
    if lse.dtype != torch.float32 or lse.shape != q.shape[:3] or lse.device != q.device:
        raise ValueError("lse must be a float32 [B, H, L] tensor on q's device")
    if out.shape != q.shape or out.dtype != q.dtype or out.stride(-1) != 1:
        raise ValueError("out must match q's shape and dtype with a contiguous last dim")
    p = _native.PartialParams()
    p.base = make_params(q, k, v, out, None, causal, scale, False, device_error_word(q.device))
    p.lse = lse.data_ptr()
    p.lse_stride[:] = (lse.stride(0), lse.stride(1), lse.stride(2))
    p.accumulate = 1 if accumulate else 0
    lib = _native.load_library()
    rc = lib.b200_attn_fwd_partial(ctypes.byref(p),
                                   ctypes.c_void_p(torch.cuda.current_stream(q.device).cuda_stream))
    if rc != _native.OK:
        raise_for_code("b200_attn_fwd_partial", rc, q.device)


def context_parallel_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                               causal: bool = True, scale: Optional[float] = None,
                               group=None) -> torch.Tensor:
    """Attention of this rank's zigzag share (``shard_sequence``) of a sequence
    sharded over the ranks of ``group``, on the sm_100a kernel; returns this
    rank's share of the output."""
    if scale is None:
        scale = q.shape[-1] ** -0.5
    out, _ = ring_attention(q, k, v, causal, scale, b200_partial_attention, group)
    return out
