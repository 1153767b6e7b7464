"""ctypes binding of the C ABI in ``include/b200_attn.h``, ``include/b200_linear.h``,
``include/b200_layernorm.h`` and ``include/b200_softmax.h``.

This module is torch-free: it loads ``libb200_attention.so`` and describes the
parameter struct.  The library is loaded from this directory only; a missing or
stale library is an error, never a reason to compute elsewhere.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libb200_attention.so"

DTYPE_BF16 = 0
DTYPE_FP16 = 1
DTYPE_FP32 = 2  # attention only: TF32 products, fp32 softmax and output

OK = 0
ERR_INVALID_ARGUMENT = 1
ERR_UNSUPPORTED = 2
ERR_ALIGNMENT = 3
ERR_DEVICE = 4
ERR_LAUNCH = 5
ERR_TIMEOUT = 6
ERR_DEVICE_BOUNDS = 7
# codes with which an entry point refuses to launch because the (host) error
# word still holds an earlier launch's report
DEVICE_REPORT_CODES = (ERR_TIMEOUT, ERR_DEVICE_BOUNDS)

DEVERR_WAIT_TIMEOUT = 1
DEVERR_BOUNDS = 2

# Every symbol the header declares; the CPU test checks the library exports them.
EXPORTED_SYMBOLS = (
    "b200_attn_abi_version",
    "b200_attn_query",
    "b200_attn_check",
    "b200_attn_fwd",
    "b200_attn_error_string",
    "b200_attn_launches_per_call",
    "b200_attn_last_error_detail",
    "b200_attn_selftest_stall",
    "b200_attn_launch_count",
    "b200_attn_launch_shape",
    "b200_attn_fwd_partial",
    "b200_attn_fwd_partial_static",
)
# Every symbol ``include/b200_linear.h`` declares.
LINEAR_SYMBOLS = (
    "b200_linear_check",
    "b200_linear_fwd",
    "b200_linear_tile_n",
)

# Every symbol ``include/b200_layernorm.h`` declares.
LAYERNORM_SYMBOLS = (
    "b200_layernorm_check",
    "b200_layernorm_fwd",
)

# Every symbol ``include/b200_softmax.h`` declares.
SOFTMAX_SYMBOLS = (
    "b200_softmax_check",
    "b200_softmax_fwd",
)
SOFTMAX_MAX_SEQ = 65536

LINEAR_ACT_NONE = 0
LINEAR_ACT_GELU = 1
LINEAR_MASKED_ZERO = 0
LINEAR_MASKED_KEEP_RESIDUAL = 1


class FwdParams(ctypes.Structure):
    """Mirror of ``b200_attn_fwd_params``."""

    _fields_ = [
        ("q", ctypes.c_void_p),
        ("k", ctypes.c_void_p),
        ("v", ctypes.c_void_p),
        ("o", ctypes.c_void_p),
        ("batch", ctypes.c_int64),
        ("heads", ctypes.c_int64),
        ("seq_len", ctypes.c_int64),
        ("head_dim", ctypes.c_int64),
        ("q_stride", ctypes.c_int64 * 3),
        ("k_stride", ctypes.c_int64 * 3),
        ("v_stride", ctypes.c_int64 * 3),
        ("o_stride", ctypes.c_int64 * 3),
        ("key_mask", ctypes.c_void_p),
        ("mask_stride", ctypes.c_int64 * 2),
        ("scale", ctypes.c_float),
        ("dtype", ctypes.c_int32),
        ("causal", ctypes.c_int32),
        ("zero_masked_queries", ctypes.c_int32),
        ("error_word", ctypes.c_void_p),
    ]


class PartialParams(ctypes.Structure):
    """Mirror of ``b200_attn_partial_params``."""

    _fields_ = [
        ("base", FwdParams),
        ("lse", ctypes.c_void_p),
        ("lse_stride", ctypes.c_int64 * 3),
        ("accumulate", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
    ]


class LinearParams(ctypes.Structure):
    """Mirror of ``b200_linear_params``."""

    _fields_ = [
        ("x", ctypes.c_void_p),
        ("w", ctypes.c_void_p),
        ("bias", ctypes.c_void_p),
        ("residual", ctypes.c_void_p),
        ("row_mask", ctypes.c_void_p),
        ("y", ctypes.c_void_p),
        ("m", ctypes.c_int64),
        ("n", ctypes.c_int64),
        ("k", ctypes.c_int64),
        ("x_row_stride", ctypes.c_int64),
        ("w_row_stride", ctypes.c_int64),
        ("residual_row_stride", ctypes.c_int64),
        ("y_row_stride", ctypes.c_int64),
        ("dtype", ctypes.c_int32),
        ("activation", ctypes.c_int32),
        ("masked_rows", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
        ("error_word", ctypes.c_void_p),
    ]


class LayerNormParams(ctypes.Structure):
    """Mirror of ``b200_layernorm_params``."""

    _fields_ = [
        ("x", ctypes.c_void_p),
        ("weight", ctypes.c_void_p),
        ("bias", ctypes.c_void_p),
        ("y", ctypes.c_void_p),
        ("rows", ctypes.c_int64),
        ("cols", ctypes.c_int64),
        ("x_row_stride", ctypes.c_int64),
        ("y_row_stride", ctypes.c_int64),
        ("eps", ctypes.c_float),
        ("dtype", ctypes.c_int32),
        ("addend", ctypes.c_void_p),
        ("sum", ctypes.c_void_p),
        ("addend_row_stride", ctypes.c_int64),
        ("sum_row_stride", ctypes.c_int64),
    ]


class SoftmaxParams(ctypes.Structure):
    """Mirror of ``b200_softmax_params``."""

    _fields_ = [
        ("scores", ctypes.c_void_p),
        ("probs", ctypes.c_void_p),
        ("batch", ctypes.c_int64),
        ("heads", ctypes.c_int64),
        ("seq_len", ctypes.c_int64),
        ("key_mask", ctypes.c_void_p),
        ("mask_stride", ctypes.c_int64 * 2),
        ("scale", ctypes.c_float),
        ("dtype", ctypes.c_int32),
        ("causal", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
    ]


_lib = None
_lock = threading.Lock()


def _bind(lib: ctypes.CDLL) -> ctypes.CDLL:
    """Declare the argument and result types of every exported entry point."""
    lib.b200_attn_abi_version.restype = ctypes.c_int32
    lib.b200_attn_abi_version.argtypes = []
    lib.b200_attn_query.restype = ctypes.c_int32
    lib.b200_attn_query.argtypes = [ctypes.c_int32, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32]
    lib.b200_attn_check.restype = ctypes.c_int32
    lib.b200_attn_check.argtypes = [ctypes.POINTER(FwdParams)]
    lib.b200_attn_fwd.restype = ctypes.c_int32
    lib.b200_attn_fwd.argtypes = [ctypes.POINTER(FwdParams), ctypes.c_void_p]
    lib.b200_attn_error_string.restype = ctypes.c_char_p
    lib.b200_attn_error_string.argtypes = [ctypes.c_int32]
    lib.b200_attn_launches_per_call.restype = ctypes.c_int32
    lib.b200_attn_launches_per_call.argtypes = [ctypes.POINTER(FwdParams)]
    lib.b200_attn_last_error_detail.restype = ctypes.c_char_p
    lib.b200_attn_last_error_detail.argtypes = []
    lib.b200_attn_launch_count.restype = ctypes.c_int64
    lib.b200_attn_launch_count.argtypes = []
    lib.b200_attn_launch_shape.restype = ctypes.c_int32
    lib.b200_attn_launch_shape.argtypes = [ctypes.c_int32, ctypes.c_int64] + [
        ctypes.POINTER(ctypes.c_int32)] * 5
    lib.b200_attn_fwd_partial.restype = ctypes.c_int32
    lib.b200_attn_fwd_partial.argtypes = [ctypes.POINTER(PartialParams), ctypes.c_void_p]
    lib.b200_attn_fwd_partial_static.restype = ctypes.c_int32
    lib.b200_attn_fwd_partial_static.argtypes = [ctypes.POINTER(FwdParams), ctypes.c_int32,
                                                 ctypes.c_void_p]
    lib.b200_attn_selftest_stall.restype = ctypes.c_int32
    lib.b200_attn_selftest_stall.argtypes = [ctypes.POINTER(FwdParams), ctypes.c_int32,
                                             ctypes.c_void_p]
    lib.b200_linear_check.restype = ctypes.c_int32
    lib.b200_linear_check.argtypes = [ctypes.POINTER(LinearParams)]
    lib.b200_linear_fwd.restype = ctypes.c_int32
    lib.b200_linear_fwd.argtypes = [ctypes.POINTER(LinearParams), ctypes.c_void_p]
    lib.b200_linear_tile_n.restype = ctypes.c_int32
    lib.b200_linear_tile_n.argtypes = [ctypes.POINTER(LinearParams), ctypes.c_int32]
    lib.b200_layernorm_check.restype = ctypes.c_int32
    lib.b200_layernorm_check.argtypes = [ctypes.POINTER(LayerNormParams)]
    lib.b200_layernorm_fwd.restype = ctypes.c_int32
    lib.b200_layernorm_fwd.argtypes = [ctypes.POINTER(LayerNormParams), ctypes.c_void_p]
    lib.b200_softmax_check.restype = ctypes.c_int32
    lib.b200_softmax_check.argtypes = [ctypes.POINTER(SoftmaxParams)]
    lib.b200_softmax_fwd.restype = ctypes.c_int32
    lib.b200_softmax_fwd.argtypes = [ctypes.POINTER(SoftmaxParams), ctypes.c_void_p]
    return lib


def load_library() -> ctypes.CDLL:
    """Load the native library (once).  Raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH.name} is not built; run `python -m b200_attention.build` "
                "or __graft_entry__.build()"
            )
        _lib = _bind(ctypes.CDLL(str(LIB_PATH)))
        return _lib


def load_checked_library() -> ctypes.CDLL:
    """The bounds-checked build of the same library (tests only)."""
    path = LIB_PATH.with_name("libb200_attention_checked.so")
    if not path.exists():
        raise RuntimeError(f"{path.name} is not built; run `python -m b200_attention.build`")
    return _bind(ctypes.CDLL(str(path)))


def error_text(code: int) -> str:
    lib = load_library()
    text = lib.b200_attn_error_string(int(code)).decode()
    detail = lib.b200_attn_last_error_detail().decode()
    return f"{text} ({detail})" if detail and code in (ERR_DEVICE, ERR_LAUNCH) else text


def launch_count() -> int:
    """Kernel launches this library has issued in this process (all entry points)."""
    return int(load_library().b200_attn_launch_count())


def launch_shape(dtype: int, head_dim: int) -> dict | None:
    """The attention kernel's launch shape for (dtype, head_dim), from the C ABI."""
    vals = [ctypes.c_int32() for _ in range(5)]
    if not load_library().b200_attn_launch_shape(int(dtype), int(head_dim),
                                                 *[ctypes.byref(v) for v in vals]):
        return None
    names = ("block_m", "rows_per_cta", "block_n", "num_warps", "ring_slots")
    return {n: v.value for n, v in zip(names, vals)}
