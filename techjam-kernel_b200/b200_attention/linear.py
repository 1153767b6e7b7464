"""Linear layer with fused epilogues on the sm_100a kernel (``include/b200_linear.h``).

``b200_linear(x, weight, bias, activation=, residual=, row_mask=, masked_rows=)``
computes ``x @ weight.T + bias`` for ``x [..., K]`` and an ``nn.Linear``
weight ``[N, K]`` on the tensor cores, and folds into the same kernel the
elementwise passes the reference block runs after its GEMMs
(torch_transformer_benchmark.py:141-145, model/triton_fused_attention.py:2456-2461):

* ``activation="gelu"``: exact (erf) GELU, ``F.gelu(..., approximate="none")``;
* ``residual``: ``residual + (x @ weight.T + bias)``;
* ``row_mask`` (bool ``[...]``, True = valid row): rows whose mask is False
  become zeros (``masked_rows="zero"``, the ``masked_fill`` after ``out_proj``
  and after each block) or keep the residual row unchanged
  (``masked_rows="residual"``: ``x + out_proj(...).masked_fill(~mask, 0)``).

Each step rounds to the 16-bit element type where the unfused sequence of
tensor ops would, so the result differs from that sequence only by the GEMM's
fp32 summation order.  Inference only (no autograd); bf16 and fp16; N and K
multiples of 8.  Inputs outside that envelope raise ``ValueError`` — there is
no fallback to another implementation.
"""

from __future__ import annotations

import ctypes
import struct
from typing import Optional

import torch

from . import _native
from .fused_attention import SIXTEEN_BIT_DTYPES, device_error_word, raise_for_code

# b200_linear_params packed in one call (layout checked against the ctypes
# mirror at import): six pointers, m n k, four row strides, dtype, activation,
# masked_rows, reserved, error word.
_LINEAR_LAYOUT = struct.Struct("=6Q7q4iQ")
assert _LINEAR_LAYOUT.size == ctypes.sizeof(_native.LinearParams)
assert _native.LinearParams.error_word.offset == _LINEAR_LAYOUT.size - 8

_MASKED_ROWS = {"zero": _native.LINEAR_MASKED_ZERO,
                "residual": _native.LINEAR_MASKED_KEEP_RESIDUAL}
_ACTIVATIONS = {None: _native.LINEAR_ACT_NONE, "none": _native.LINEAR_ACT_NONE,
                "gelu": _native.LINEAR_ACT_GELU}


def linear_supported(x: torch.Tensor, weight: torch.Tensor) -> bool:
    """True when ``b200_linear`` accepts these operands (device, dtype, sizes)."""
    return (x.is_cuda and x.dtype in SIXTEEN_BIT_DTYPES and weight.dtype == x.dtype
            and weight.device == x.device and weight.dim() == 2
            and weight.shape[1] == x.shape[-1] and weight.shape[0] % 8 == 0
            and weight.shape[1] % 8 == 0)


def _rows(t: torch.Tensor, cols: int) -> torch.Tensor:
    """``t`` as a 2-D [rows, cols] view with a contiguous last dim and
    non-overlapping rows whose stride is a multiple of 8 elements (copied only
    when no such view exists, e.g. for a broadcast ``expand``)."""
    flat = t.reshape(-1, cols)
    if (flat.stride(-1) != 1
            or (flat.shape[0] > 1 and (flat.stride(0) % 8 != 0 or flat.stride(0) < cols))
            or flat.data_ptr() % 16 != 0):
        flat = flat.contiguous()
    return flat


def b200_linear(
    x: torch.Tensor,
    weight: torch.Tensor,
    bias: Optional[torch.Tensor] = None,
    *,
    activation: Optional[str] = None,
    residual: Optional[torch.Tensor] = None,
    row_mask: Optional[torch.Tensor] = None,
    masked_rows: str = "zero",
) -> torch.Tensor:
    """``epilogue(x @ weight.T + bias)`` on the sm_100a kernel; a new tensor
    ``[..., N]`` in ``x``'s dtype.  See the module docstring for the epilogue."""
    if activation not in _ACTIVATIONS:
        raise ValueError(f"activation must be None or 'gelu', got {activation!r}")
    if masked_rows not in _MASKED_ROWS:
        raise ValueError(f"masked_rows must be 'zero' or 'residual', got {masked_rows!r}")
    if x.dim() < 1 or weight.dim() != 2:
        raise ValueError("x must be [..., K] and weight [N, K]")
    n, k = weight.shape
    if x.shape[-1] != k:
        raise ValueError(f"x has {x.shape[-1]} features, weight expects {k}")
    if x.dtype not in SIXTEEN_BIT_DTYPES:
        raise ValueError(f"b200_linear supports bfloat16 and float16, got {x.dtype}")
    tensors = [("weight", weight), ("bias", bias), ("residual", residual)]
    for name, t in tensors:
        if t is None:
            continue
        if t.dtype != x.dtype:
            raise TypeError(f"{name} must have x's dtype {x.dtype}, got {t.dtype}")
        if t.device != x.device:
            raise ValueError(f"{name} must be on x's device")
    if bias is not None and tuple(bias.shape) != (n,):
        raise ValueError(f"bias must have shape ({n},)")
    lead = tuple(x.shape[:-1])
    if residual is not None and tuple(residual.shape) != lead + (n,):
        raise ValueError(f"residual must have shape {lead + (n,)}")
    if row_mask is not None:
        if row_mask.dtype != torch.bool:
            raise TypeError("row_mask must have dtype torch.bool")
        if tuple(row_mask.shape) != lead or row_mask.device != x.device:
            raise ValueError(f"row_mask must be a bool tensor of shape {lead} on x's device")
        if masked_rows == "residual" and residual is None:
            raise ValueError("masked_rows='residual' needs a residual")
    if n % 8 or k % 8:
        raise ValueError("b200_linear needs N and K to be multiples of 8")
    if torch.is_grad_enabled() and any(t is not None and t.requires_grad
                                       for t in (x, weight, bias, residual)):
        raise ValueError("b200_linear is inference-only: it records no autograd graph")
    if not x.is_cuda:
        raise ValueError("b200_linear runs on CUDA tensors only")

    y = torch.empty(lead + (n,), device=x.device, dtype=x.dtype)
    if y.numel() == 0:
        return y
    x2 = _rows(x, k)
    w2 = _rows(weight, k)
    b1 = None
    if bias is not None:
        b1 = bias if bias.is_contiguous() and bias.data_ptr() % 16 == 0 else bias.clone(
            memory_format=torch.contiguous_format)
    r2 = None if residual is None else _rows(residual, n)
    m1 = None if row_mask is None else row_mask.reshape(-1).contiguous()
    y2 = y.view(-1, n)

    p = _native.LinearParams()
    _LINEAR_LAYOUT.pack_into(
        p, 0, x2.data_ptr(), w2.data_ptr(), b1.data_ptr() if b1 is not None else 0,
        r2.data_ptr() if r2 is not None else 0, m1.data_ptr() if m1 is not None else 0,
        y2.data_ptr(), x2.shape[0], n, k, x2.stride(0), w2.stride(0),
        r2.stride(0) if r2 is not None else 0, y2.stride(0), SIXTEEN_BIT_DTYPES[x.dtype],
        _ACTIVATIONS[activation], _MASKED_ROWS[masked_rows], 0,
        device_error_word(x.device).data_ptr())

    lib = _native.load_library()
    stream = torch.cuda.current_stream(x.device).cuda_stream
    rc = lib.b200_linear_fwd(ctypes.byref(p), ctypes.c_void_p(stream))
    if rc != _native.OK:
        raise_for_code("b200_linear_fwd", rc, x.device)
    return y
