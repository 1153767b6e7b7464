"""The allocation-free context-parallel step, ``b200_attn_fwd_partial_static``.

Some callers of this library cannot call cudaMalloc: a serving host whose
memory pool has already taken the device's memory, a latency-bound loop that
cannot take the device-wide synchronisation cudaMalloc and cudaFree bring, or
a binding from another language with no device allocator.  For them the
entry point keeps the per-row log-sum-exp, which carries a query chunk's merge
from one call to the next, in a fixed array inside the library.

The GPU test runs one query chunk over two key chunks (a first call, then an
accumulating call), twice in a row with different shapes and dtypes, through
the C ABI.  Each result is compared with ``b200_attn_fwd_partial`` given a
log-sum-exp tensor of its own, within the tolerance of every other parity test
(max-abs <= 2e-2, mean-abs <= 2e-3), and with the oracle over the whole
sequence.  This file is named to be collected last.
"""

import ctypes

import pytest
import torch

from b200_attention import _native, read_device_errors
from b200_attention.context_parallel import b200_partial_attention
from b200_attention.fused_attention import device_error_word, make_params
from oracle.reference_attention import reference_attention
from parity import assert_close, seeded_qkv

MAX_ROWS = 1 << 20  # B200_ATTN_STATIC_LSE_MAX_ROWS


def _static_step(lib, q, k, v, out, causal, scale, accumulate, word):
    p = make_params(q, k, v, out, None, causal, scale, False, word)
    stream = ctypes.c_void_p(torch.cuda.current_stream(q.device).cuda_stream)
    return lib.b200_attn_fwd_partial_static(ctypes.byref(p), 1 if accumulate else 0, stream)


def _second_half(q, k, v, L):
    """The query chunk (rows L..2L) and the two key chunks it sees."""
    return (q[:, :, L:].contiguous(), k[:, :, :L].contiguous(), v[:, :, :L].contiguous(),
            k[:, :, L:].contiguous(), v[:, :, L:].contiguous())


@pytest.mark.gpu
def test_static_partial_matches_partial_on_two_calls_in_a_row():
    dev = torch.device("cuda", 0)
    lib = _native.load_library()
    word = device_error_word(dev)
    cases = [((2, 4, 2 * 384, 128), torch.bfloat16, 31), ((1, 3, 2 * 200, 64), torch.float16, 32)]
    for shape, dtype, seed in cases:
        B, H, S, D = shape
        L, scale = S // 2, D ** -0.5
        q, k, v = seeded_qkv(shape, dtype, seed)
        qc, k0, v0, k1, v1 = (t.to(dev) for t in _second_half(q, k, v, L))

        # existing entry point, with a log-sum-exp tensor of its own
        want = torch.empty_like(qc)
        lse = torch.empty((B, H, L), device=dev, dtype=torch.float32)
        b200_partial_attention(qc, k0, v0, False, scale, want, lse, False)
        b200_partial_attention(qc, k1, v1, True, scale, want, lse, True)

        # allocation-free entry point: the same two calls, no log-sum-exp buffer
        got = torch.full_like(qc, float("nan"))
        assert _static_step(lib, qc, k0, v0, got, False, scale, False, word) == _native.OK
        assert _static_step(lib, qc, k1, v1, got, True, scale, True, word) == _native.OK
        torch.cuda.synchronize(dev)
        assert read_device_errors(dev) == 0

        label = f"static partial {dtype} {shape}"
        assert_close(got.cpu(), want.cpu(), label)
        ref = reference_attention(q, k, v, None, True, scale)[:, :, L:]
        assert_close(got.cpu(), ref, label + " vs oracle")


@pytest.mark.gpu
def test_static_partial_refuses_an_unmatched_accumulating_call():
    dev = torch.device("cuda", 0)
    lib = _native.load_library()
    word = device_error_word(dev)
    q, k, v = (t.to(dev) for t in seeded_qkv((1, 2, 256, 64), torch.bfloat16, 33))
    out = torch.empty_like(q)
    assert _static_step(lib, q, k, v, out, True, 0.125, False, word) == _native.OK
    # an accumulating call of another shape would merge into rows it never wrote
    q2, k2, v2 = (t[:, :1].contiguous() for t in (q, k, v))
    before = _native.launch_count()
    rc = _static_step(lib, q2, k2, v2, torch.empty_like(q2), True, 0.125, True, word)
    assert rc == _native.ERR_INVALID_ARGUMENT
    assert _native.launch_count() == before
    torch.cuda.synchronize(dev)
    assert read_device_errors(dev) == 0


def test_static_partial_rejects_more_rows_than_its_array_holds():
    """Host-side size check: runs before any CUDA call, so it needs no GPU."""
    lib = _native.load_library()
    p = _native.FwdParams()
    p.q = p.k = p.v = p.o = 1 << 20  # never dereferenced: refused first
    p.batch, p.heads, p.head_dim = 1, 32, 64
    p.seq_len = MAX_ROWS // 32 + 1
    for st in (p.q_stride, p.k_stride, p.v_stride, p.o_stride):
        st[0], st[1], st[2] = 32 * p.seq_len * 64, p.seq_len * 64, 64
    p.scale, p.dtype, p.causal = 0.125, _native.DTYPE_BF16, 1
    assert lib.b200_attn_check(ctypes.byref(p)) == _native.OK
    assert lib.b200_attn_fwd_partial_static(ctypes.byref(p), 0, None) == _native.ERR_INVALID_ARGUMENT
    assert b"B200_ATTN_STATIC_LSE_MAX_ROWS" in lib.b200_attn_last_error_detail()
    p.seq_len = MAX_ROWS // 32
    assert lib.b200_attn_check(ctypes.byref(p)) == _native.OK
