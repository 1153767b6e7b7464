"""Bounds-checked build on odd shapes (the stand-in for a sanitizer, which is
closed on this pool).

``libb200_attention_checked.so`` is the same kernel source compiled with every
TMA coordinate, shared-memory tile address and tensor-memory column range
verified on the device; a failed check sets ``B200_ATTN_DEVERR_BOUNDS`` in the
error word and skips the access.  Each case must leave the word clear and match
the oracle.
"""

import ctypes

import pytest
import torch

from b200_attention import _native
from b200_attention.fused_attention import device_error_word, make_params, read_device_errors
from oracle.reference_attention import reference_attention, zero_masked_rows
from parity import assert_close, prefix_mask, seeded_qkv

pytestmark = pytest.mark.gpu

CASES = [
    # (B, H, S, D, causal, lengths, zero_masked_queries)
    (1, 1, 1, 128, True, None, False),
    (2, 2, 33, 64, False, None, False),
    (1, 3, 97, 128, True, None, False),
    (2, 1, 129, 64, True, None, False),
    (1, 2, 255, 128, False, None, False),
    (2, 2, 257, 128, True, [257, 100], False),
    (3, 2, 700, 64, False, [700, 333, 1], True),
    (1, 2, 1000, 128, True, None, False),
    (2, 1, 1536, 128, False, [1536, 700], True),
    # narrow heads: the 64- / 128-wide instance reads zeros past the head dim
    (2, 2, 300, 32, True, [300, 123], True),
    (1, 3, 129, 8, False, None, False),
    (2, 1, 257, 96, True, None, False),
]


# fp32 inputs (TF32 products) on the fp32 instance: head dims up to 64
CASES_FP32 = [
    (1, 1, 1, 64, True, None, False),
    (2, 2, 33, 64, False, None, False),
    (2, 1, 129, 64, True, None, False),
    (3, 2, 700, 64, False, [700, 333, 1], True),
    (1, 2, 1000, 64, True, None, False),
    (2, 2, 300, 32, True, [300, 123], True),
    (1, 3, 129, 8, False, None, False),
    (2, 1, 257, 40, True, None, False),
]


def _case_id(c):
    dtype, B, H, S, D, causal, lengths, zero_q = c
    return f"{str(dtype).removeprefix('torch.')}-B{B}H{H}S{S}D{D}{'-causal' if causal else ''}" \
           f"{'-mask' if lengths else ''}{'-zeroq' if zero_q else ''}"


_ALL = [(torch.bfloat16, *c) for c in CASES] + [(torch.float32, *c) for c in CASES_FP32]


@pytest.mark.parametrize("dtype,B,H,S,D,causal,lengths,zero_q", _ALL, ids=[_case_id(c) for c in _ALL])
def test_checked_build_odd_shapes(dtype, B, H, S, D, causal, lengths, zero_q):
    dev = torch.device("cuda", 0)
    lib = _native.load_checked_library()
    q, k, v = seeded_qkv((B, H, S, D), dtype, 41 + S)
    mask = prefix_mask(B, S, lengths) if lengths else None
    qd, kd, vd = q.to(dev), k.to(dev), v.to(dev)
    md = mask.to(dev) if mask is not None else None
    out = torch.full((B, H, S, D), float("nan"), device=dev, dtype=dtype)
    read_device_errors(dev)
    params = make_params(qd, kd, vd, out, md, causal, D ** -0.5, zero_q, device_error_word(dev))
    rc = lib.b200_attn_fwd(ctypes.byref(params),
                           ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream))
    assert rc == _native.OK
    torch.cuda.synchronize(dev)
    assert read_device_errors(dev) == 0, "a bounds check failed"
    ref = reference_attention(q, k, v, mask, causal, D ** -0.5)
    if zero_q:
        ref = zero_masked_rows(ref, mask)
    assert_close(out, ref, f"checked {dtype} B{B} H{H} S{S} D{D}")


@pytest.mark.parametrize("dtype,D", [(torch.bfloat16, 128), (torch.float16, 64), (torch.float32, 64)])
def test_checked_build_partial_form(dtype, D):
    """The context-parallel partial instances in the bounds-checked build: a
    diagonal chunk, then an earlier chunk merged in (accumulate); the word
    stays clear and the merge equals attention over both chunks."""
    dev = torch.device("cuda", 0)
    lib = _native.load_checked_library()
    L = 300
    q, k, v = seeded_qkv((1, 2, 2 * L, D), dtype, 91)
    qd, kd, vd = q.to(dev), k.to(dev), v.to(dev)
    out = torch.empty((1, 2, L, D), device=dev, dtype=dtype)
    lse = torch.empty((1, 2, L), device=dev, dtype=torch.float32)
    read_device_errors(dev)
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    for k_lo, causal, acc in ((L, True, 0), (0, False, 1)):  # query chunk = rows L..2L
        pp = _native.PartialParams()
        pp.base = make_params(qd[:, :, L:], kd[:, :, k_lo:k_lo + L], vd[:, :, k_lo:k_lo + L], out,
                              None, causal, D ** -0.5, False, device_error_word(dev))
        pp.lse = lse.data_ptr()
        pp.lse_stride[:] = (lse.stride(0), lse.stride(1), lse.stride(2))
        pp.accumulate = acc
        assert lib.b200_attn_fwd_partial(ctypes.byref(pp), stream) == _native.OK
    torch.cuda.synchronize(dev)
    assert read_device_errors(dev) == 0, "a bounds check failed"
    ref = reference_attention(q, k, v, None, True, D ** -0.5)[:, :, L:]
    assert_close(out, ref, f"checked partial {dtype}")
