"""Failure detection on the GPU without a GPU fault.

The self-test entry point ``b200_attn_selftest_stall`` launches the real
kernel with one K/V load of every CTA announced to its barrier but never
issued (a flag that nothing sets).  The pipeline wait on it must run out
after its one-second bound, the kernel must report
``B200_ATTN_DEVERR_WAIT_TIMEOUT`` in the error word and return on its own,
and the CUDA context must stay usable: the next ordinary call is correct and
reports no error.  No trap, no device assert, no bad address, no endless loop.
"""

import ctypes
import time

import pytest
import torch

from b200_attention import _native
from b200_attention.fused_attention import (b200_fused_attention, device_error_word, make_params,
                                            read_device_errors)
from oracle.reference_attention import reference_attention
from parity import assert_close, seeded_qkv

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("skipped_load", [0, 3])
def test_stalled_pipeline_reports_timeout_and_context_survives(skipped_load):
    dev = torch.device("cuda", 0)
    q, k, v = seeded_qkv((1, 2, 512, 128), torch.bfloat16, 31)
    qd, kd, vd = q.to(dev), k.to(dev), v.to(dev)
    out = torch.empty_like(qd)
    read_device_errors(dev)  # start clean
    word = device_error_word(dev)
    params = make_params(qd, kd, vd, out, None, True, 128 ** -0.5, False, word)
    lib = _native.load_library()
    stream = torch.cuda.current_stream(dev).cuda_stream
    t0 = time.perf_counter()
    rc = lib.b200_attn_selftest_stall(ctypes.byref(params), skipped_load, ctypes.c_void_p(stream))
    assert rc == _native.OK
    torch.cuda.synchronize(dev)
    elapsed = time.perf_counter() - t0
    assert read_device_errors(dev) & _native.DEVERR_WAIT_TIMEOUT
    assert 0.5 < elapsed < 30.0, elapsed  # bounded waits, not a hang

    ref = reference_attention(q, k, v, None, True, 128 ** -0.5)
    assert_close(b200_fused_attention(qd, kd, vd, None, True), ref, "after the stall")
    torch.cuda.synchronize(dev)
    assert read_device_errors(dev) == 0


def test_selftest_rejects_configurations_it_does_not_cover():
    dev = torch.device("cuda", 0)
    q = torch.zeros((1, 1, 128, 64), device=dev, dtype=torch.bfloat16)
    params = make_params(q, q, q, torch.empty_like(q), None, True, 0.125, False,
                         device_error_word(dev))
    lib = _native.load_library()
    assert lib.b200_attn_selftest_stall(ctypes.byref(params), 0, None) == _native.ERR_UNSUPPORTED


def test_module_and_decoder_raise_after_a_device_reported_timeout():
    """After a launch reports a pipeline timeout in the device's error word,
    the operator, the module and the decoder raise DeviceError instead of
    returning a tensor (the C ABI refuses to launch while the host-visible word
    holds the report); clearing the word resumes normal, correct launches."""
    from b200_attention import DeviceError, check_device_errors, clear_device_errors
    from b200_attention.modules import B200FusedSelfAttention
    from b200_attention.transformer import Decoder, DecoderConfig, init_normal_

    dev = torch.device("cuda", 0)
    clear_device_errors(dev)
    q, k, v = (t.to(dev) for t in seeded_qkv((1, 2, 512, 128), torch.bfloat16, 37))
    params = make_params(q, k, v, torch.empty_like(q), None, True, 128 ** -0.5, False,
                         device_error_word(dev))
    lib = _native.load_library()
    rc = lib.b200_attn_selftest_stall(ctypes.byref(params), 1,
                                      ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream))
    assert rc == _native.OK
    torch.cuda.synchronize(dev)  # the stalled launch has finished and reported

    module = B200FusedSelfAttention(256, 4).to(dev, torch.bfloat16).eval()
    decoder = init_normal_(Decoder(DecoderConfig(2, 128, 256, 4, 512, 2, True)), seed=3)
    decoder = decoder.to(dev, torch.bfloat16).eval()
    x = torch.randn(2, 128, 256, device=dev, dtype=torch.bfloat16)
    with torch.inference_mode():
        with pytest.raises(DeviceError, match="timeout"):
            check_device_errors(dev)
        with pytest.raises(DeviceError, match="refused to launch"):
            b200_fused_attention(q, k, v, None, True)
        with pytest.raises(DeviceError):
            module(x, None, causal=True)
        with pytest.raises(DeviceError):
            decoder(x)
        clear_device_errors(dev)
        check_device_errors(dev)
        ref = reference_attention(q.cpu(), k.cpu(), v.cpu(), None, True, 128 ** -0.5)
        assert_close(b200_fused_attention(q, k, v, None, True), ref, "after clearing")
        assert torch.isfinite(decoder(x).float()).all()
    assert read_device_errors(dev) == 0
