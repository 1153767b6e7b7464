"""Functional attention operator over the sm_100a kernel.

``b200_fused_attention`` keeps the signature, argument meaning and error
behaviour of the reference operator ``triton_fused_attention``
(model/triton_fused_attention.py:1877-1891): ``q, k, v`` are ``[B, H, S, D]``
tensors with a contiguous last dimension (transposed projection views are
consumed through their strides), ``valid_token_mask`` is an optional bool
``[B, S]`` key mask, ``causal`` is top-left aligned, ``scale`` defaults to
``D ** -0.5`` and must be positive, and ``output_bshd`` selects a contiguous
``[B, S, H, D]`` output instead of ``[B, H, S, D]``.

The call is one torch custom op over the C ABI (``csrc/torch_op.cpp``);
``make_params`` packs the same C struct for callers that use the C ABI
directly (the self-test and bounds-checked entry points).

One deliberate difference: the reference silently falls back to dense PyTorch
for inputs its kernels do not cover (:1906-1925).  This operator has no fallback
of any kind; inputs outside the kernel envelope raise ``ValueError`` whatever
``strict`` says.  Choosing an exact PyTorch path for such inputs is the
planner's decision (``attention_dispatch``), made visibly, not the operator's.
"""

from __future__ import annotations

import ctypes
import struct
import threading
from typing import Optional

import torch

from . import _native

# Element types of the block's linear and LayerNorm kernels (16-bit only).
SIXTEEN_BIT_DTYPES = {torch.bfloat16: _native.DTYPE_BF16, torch.float16: _native.DTYPE_FP16}
# Element types of the attention kernel: fp32 inputs run the fp32 instance,
# whose products are TF32 (the reference's fp32 tiled kernel's precision,
# model/triton_fused_attention.py:235-356) with an fp32 softmax and output.
SUPPORTED_DTYPES = {**SIXTEEN_BIT_DTYPES, torch.float32: _native.DTYPE_FP32}
# Every multiple of 8 up to 128.  The kernel's 64- and 128-wide instances read
# the missing columns of narrower heads as zeros through TMA (zero columns add
# nothing to Q K^T and P V) and its output store clips them; the softmax scale
# stays that of the true head dim.  No padded copies are made.
SUPPORTED_HEAD_DIMS = tuple(range(8, 129, 8))
# fp32: multiples of 8 up to 64 (one 64-wide fp32 instance)
FP32_HEAD_DIMS = tuple(range(8, 65, 8))
NATIVE_HEAD_DIMS = SUPPORTED_HEAD_DIMS
BLOCK_M = 128  # query rows per tile (two tiles per CTA)
BLOCK_N = 128  # keys per K/V tile

_error_words: dict[int, torch.Tensor] = {}
_error_lock = threading.Lock()


def _validate_inputs(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    valid_token_mask: Optional[torch.Tensor],
) -> tuple[int, int, int, int]:
    """Common tensor contract; same checks and exception types as the reference
    (model/triton_fused_attention.py:1217-1253)."""
    if q.ndim != 4:
        raise ValueError(f"q must have shape [B, H, S, D], got {tuple(q.shape)}")
    if k.shape != q.shape or v.shape != q.shape:
        raise ValueError(
            "q, k, and v must have the same [B, H, S, D] shape; "
            f"got q={tuple(q.shape)}, k={tuple(k.shape)}, v={tuple(v.shape)}"
        )
    if q.device != k.device or q.device != v.device:
        raise ValueError("q, k, and v must be on the same device")
    if q.dtype != k.dtype or q.dtype != v.dtype:
        raise TypeError("q, k, and v must have the same dtype")
    if not q.dtype.is_floating_point:
        raise TypeError(f"q/k/v must use a floating-point dtype, got {q.dtype}")
    batch, heads, seq_len, head_dim = q.shape
    if seq_len <= 0 or head_dim <= 0:
        raise ValueError("sequence length and head dimension must be positive")
    if valid_token_mask is not None:
        if valid_token_mask.shape != (batch, seq_len):
            raise ValueError(
                "valid_token_mask must have shape "
                f"{(batch, seq_len)}, got {tuple(valid_token_mask.shape)}"
            )
        if valid_token_mask.dtype != torch.bool:
            raise TypeError("valid_token_mask must have dtype torch.bool")
        if valid_token_mask.device != q.device:
            raise ValueError("valid_token_mask and q must be on the same device")
    return batch, heads, seq_len, head_dim


def unsupported_reason(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> Optional[str]:
    """Why the sm_100a kernel cannot run these inputs, or None when it can."""
    if q.device.type != "cuda":
        return "inputs must be CUDA tensors"
    if q.dtype not in SUPPORTED_DTYPES:
        return f"dtype {q.dtype} is outside the kernel envelope (bfloat16, float16, float32)"
    if q.dtype == torch.float32 and q.shape[-1] not in FP32_HEAD_DIMS:
        return (f"head_dim {q.shape[-1]} is outside the kernel envelope for float32 "
                "(multiples of 8 up to 64)")
    if q.shape[-1] not in SUPPORTED_HEAD_DIMS:
        return (f"head_dim {q.shape[-1]} is outside the kernel envelope "
                "(multiples of 8 up to 128)")
    if q.stride(-1) != 1 or k.stride(-1) != 1 or v.stride(-1) != 1:
        return "q/k/v must have a contiguous last dimension"
    if torch.is_grad_enabled() and (q.requires_grad or k.requires_grad or v.requires_grad):
        return "the kernel is inference-only (autograd requested)"
    major = _capability_major(q.device)
    if major != 10:
        return f"the kernel is built for sm_100a; device capability is {major}.x"
    return None


_capability: dict = {}


def _capability_major(device: torch.device) -> int:
    index = device.index if device.index is not None else torch.cuda.current_device()
    major = _capability.get(index)
    if major is None:
        major = _capability[index] = torch.cuda.get_device_capability(index)[0]
    return major


class DeviceError(RuntimeError):
    """A kernel launched earlier on this device reported an error (a pipeline
    wait that ran out, or a failed bounds check in the checked build) in the
    device's error word.  The outputs of that launch are undefined; every later
    launch on the device is refused until ``clear_device_errors`` is called."""


_DEVERR_NAMES = {_native.DEVERR_WAIT_TIMEOUT: "pipeline wait timeout",
                 _native.DEVERR_BOUNDS: "failed bounds check"}


def _describe(bits: int) -> str:
    names = [name for bit, name in _DEVERR_NAMES.items() if bits & bit]
    return ", ".join(names) or f"error bits {bits:#x}"


def device_error_word(device: torch.device) -> torch.Tensor:
    """Per-device int32 error word that every kernel of this package reports
    into (allocated once).  It lives in pinned host memory the device
    addresses directly, so the host can read it without synchronising: each
    entry point checks it before launching and refuses to launch while it
    holds a report (``include/b200_attn.h``, "Error word")."""
    index = device.index if device.index is not None else torch.cuda.current_device()
    word = _error_words.get(index)
    if word is None:
        with _error_lock:
            word = _error_words.get(index)
            if word is None:
                # a normal tensor even when the first call runs under
                # torch.inference_mode(), so the word can be cleared anywhere
                with torch.inference_mode(False):
                    word = torch.zeros(1, dtype=torch.int32, pin_memory=True)
                _error_words[index] = word
    return word


def read_device_errors(device: torch.device, clear: bool = True) -> int:
    """Synchronise ``device`` and return the error bits its kernels reported
    (clearing them unless ``clear`` is False)."""
    word = device_error_word(device)
    torch.cuda.synchronize(device)
    value = int(word[0])
    if clear and value:
        word.zero_()
    return value


def clear_device_errors(device: torch.device) -> None:
    """Synchronise ``device`` and clear its error word (launches resume)."""
    read_device_errors(device, clear=True)


def check_device_errors(device: torch.device) -> None:
    """Raise ``DeviceError`` when a launch that already finished on ``device``
    reported an error.  Reads the host-side word only: no synchronisation,
    safe inside CUDA graph capture."""
    value = int(device_error_word(device)[0])
    if value:
        raise DeviceError(f"a kernel on {device} reported a {_describe(value)}; its output is "
                          "undefined (clear_device_errors resumes launches)")


def raise_for_code(entry: str, rc: int, device: torch.device) -> None:
    """Turn a nonzero C-ABI return code into the exception the reference's
    operator raises for it (``ValueError`` for contract violations)."""
    if rc in (_native.ERR_INVALID_ARGUMENT, _native.ERR_ALIGNMENT):
        raise ValueError(f"{entry}: {_native.error_text(rc)}")
    if rc == _native.ERR_UNSUPPORTED:
        raise ValueError(f"unsupported sm_100a invocation ({entry}): {_native.error_text(rc)}")
    if rc in _native.DEVICE_REPORT_CODES:
        value = int(device_error_word(device)[0])
        raise DeviceError(f"{entry} refused to launch: an earlier kernel on {device} reported a "
                          f"{_describe(value)}; its output is undefined "
                          "(clear_device_errors resumes launches)")
    raise RuntimeError(f"{entry}: {_native.error_text(rc)}")


def _strides(t: torch.Tensor) -> tuple[int, int, int]:
    return (t.stride(0), t.stride(1), t.stride(2))


# b200_attn_fwd_params packed in one call (layout checked against the ctypes
# mirror at import): q k v o, B H S D, four stride triples, mask and its two
# strides, scale, dtype, causal, zero_masked_queries, error word.
_FWD_LAYOUT = struct.Struct("=4Q4q12qQ2qfiiiQ")
assert _FWD_LAYOUT.size == ctypes.sizeof(_native.FwdParams)
assert _native.FwdParams.error_word.offset == _FWD_LAYOUT.size - 8


def make_params(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    out_bhsd: torch.Tensor,
    valid_token_mask: Optional[torch.Tensor],
    causal: bool,
    scale: float,
    zero_masked_queries: bool,
    error_word: Optional[torch.Tensor],
) -> _native.FwdParams:
    """Fill the C parameter struct from tensors (``out_bhsd`` is a [B,H,S,D] view)."""
    p = _native.FwdParams()
    if valid_token_mask is not None:
        mask, ms0, ms1 = (valid_token_mask.data_ptr(), valid_token_mask.stride(0),
                          valid_token_mask.stride(1))
    else:
        mask = ms0 = ms1 = 0
    _FWD_LAYOUT.pack_into(
        p, 0, q.data_ptr(), k.data_ptr(), v.data_ptr(), out_bhsd.data_ptr(), *q.shape,
        *q.stride()[:3], *k.stride()[:3], *v.stride()[:3], *out_bhsd.stride()[:3],
        mask, ms0, ms1, float(scale), SUPPORTED_DTYPES[q.dtype], 1 if causal else 0,
        1 if zero_masked_queries else 0, error_word.data_ptr() if error_word is not None else 0)
    return p


_op = None
_op_lock = threading.Lock()
_word_ptrs: dict = {}


def _attention_op():
    """torch.ops.b200.fused_attention, loaded once from this directory.  Raises
    when the library has not been built; there is no other implementation."""
    global _op
    if _op is None:
        with _op_lock:
            if _op is None:
                from .build import TORCH_OP_PATH

                if not TORCH_OP_PATH.exists():
                    raise RuntimeError(f"{TORCH_OP_PATH.name} is not built; run "
                                       "`python -m b200_attention.build` or __graft_entry__.build()")
                _native.load_library()
                torch.ops.load_library(str(TORCH_OP_PATH))
                _op = torch.ops.b200.fused_attention
    return _op


def _error_word_address(device: torch.device) -> int:
    address = _word_ptrs.get(device)
    if address is None:
        address = _word_ptrs[device] = (device_error_word(device).data_ptr()
                                        if device.type == "cuda" else 0)
    return address


def b200_fused_attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    valid_token_mask: Optional[torch.Tensor] = None,
    causal: bool = False,
    scale: Optional[float] = None,
    output_bshd: bool = False,
    *,
    strict: bool = False,
    block_m: Optional[int] = None,
    block_n: Optional[int] = None,
    num_warps: Optional[int] = None,
    num_stages: Optional[int] = None,
    zero_masked_queries: bool = False,
    out: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """Attention forward on the sm_100a kernel without materialising S x S.

    Returns a new ``[B, H, S, D]`` tensor (or contiguous ``[B, S, H, D]`` with
    ``output_bshd``).  ``zero_masked_queries`` additionally writes zeros for query
    rows whose own mask bit is False (the value the reference's module produces
    for them after its output projection, :2460-2461); it skips all work for
    query blocks that lie entirely past the last valid key.  ``out`` may supply
    the output tensor (same shape/dtype/device, contiguous last dim).

    The call is one torch custom op (``torch.ops.b200.fused_attention``,
    ``csrc/torch_op.cpp``) over the C ABI: the reference's input checks with
    its exception types, the output allocation and the launch on the current
    stream happen in C++.  ``block_m``/``block_n`` are accepted for signature
    compatibility; the kernel uses fixed 128 x 128 tiles and rejects other
    values.  ``num_warps`` and ``num_stages`` are accepted and ignored (the
    kernel's warp roles and ring depth are fixed per head dimension).
    ``strict`` is accepted; unsupported inputs always raise.
    """
    if block_m not in (None, BLOCK_M) or block_n not in (None, BLOCK_N):
        raise ValueError(f"the sm_100a kernel uses {BLOCK_M}x{BLOCK_N} tiles")
    op = _op if _op is not None else _attention_op()
    try:
        return op(q, k, v, valid_token_mask, causal, scale, output_bshd, zero_masked_queries, out,
                  _error_word_address(q.device))
    except RuntimeError as exc:
        if str(exc).startswith("b200 device error"):
            value = int(device_error_word(q.device)[0])
            raise DeviceError(f"b200_attn_fwd refused to launch: an earlier kernel on {q.device} "
                              f"reported a {_describe(value)}; its output is undefined "
                              "(clear_device_errors resumes launches)") from None
        raise
