"""LayerNorm over the last dimension on the B200 (``include/b200_layernorm.h``).

``b200_layer_norm(x, weight, bias, eps)`` has the semantics of
``F.layer_norm(x, (x.shape[-1],), weight, bias, eps)`` (biased variance; mean,
variance and the affine step in fp32, one rounding to the element type) for
bf16/fp16 inputs whose last dimension is a multiple of 8 up to 4096.  It
replaces the reference block's norm1/norm2 and the model's final norm
(torch_transformer_benchmark.py:141-142, 170) in the decoder's fused path;
``b200_add_layer_norm`` also forms the residual sum that precedes the norm.
Inference only; anything outside the envelope raises ``ValueError``.
"""

from __future__ import annotations

import ctypes
import struct
from typing import Optional

import torch

from . import _native
from .fused_attention import SIXTEEN_BIT_DTYPES, raise_for_code

MAX_COLS = 4096

# b200_layernorm_params packed in one call (layout checked against the ctypes
# mirror at import): x weight bias y, rows cols and the two row strides, eps,
# dtype, addend and sum pointers and their row strides.
_LN_LAYOUT = struct.Struct("=4Q4qfi2Q2q")
assert _LN_LAYOUT.size == ctypes.sizeof(_native.LayerNormParams)


def layer_norm_supported(x: torch.Tensor, weight: Optional[torch.Tensor]) -> bool:
    cols = x.shape[-1]
    return (x.is_cuda and x.dtype in SIXTEEN_BIT_DTYPES and cols % 8 == 0 and 0 < cols <= MAX_COLS
            and (weight is None or (weight.dtype == x.dtype and weight.device == x.device)))


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


def _vector(t: Optional[torch.Tensor], cols: int, name: str, x: torch.Tensor):
    if t is None:
        return None
    if tuple(t.shape) != (cols,):
        raise ValueError(f"{name} must have shape ({cols},)")
    if t.dtype != x.dtype:
        raise TypeError(f"{name} must have x's dtype {x.dtype}, got {t.dtype}")
    if t.device != x.device:
        raise ValueError(f"{name} must be on x's device")
    if not t.is_contiguous() or t.data_ptr() % 16 != 0:
        t = t.clone(memory_format=torch.contiguous_format)
    return t


def b200_layer_norm(x: torch.Tensor, weight: Optional[torch.Tensor] = None,
                    bias: Optional[torch.Tensor] = None, eps: float = 1e-5) -> torch.Tensor:
    """LayerNorm of ``x`` over its last dimension; a new tensor like ``x``."""
    return _layer_norm(x, None, weight, bias, eps)[1]


def b200_add_layer_norm(x: torch.Tensor, addend: torch.Tensor,
                        weight: Optional[torch.Tensor] = None,
                        bias: Optional[torch.Tensor] = None,
                        eps: float = 1e-5) -> tuple[torch.Tensor, torch.Tensor]:
    """``(s, LayerNorm(s))`` for the residual sum ``s = x + addend`` (rounded
    once to the element type, as a 16-bit tensor add is), in one pass: the
    residual add that ends one reference block and the norm that starts the
    next (torch_transformer_benchmark.py:141-142) or the final norm (:170)."""
    if tuple(addend.shape) != tuple(x.shape):
        raise ValueError(f"addend must have x's shape {tuple(x.shape)}")
    if addend.dtype != x.dtype:
        raise TypeError(f"addend must have x's dtype {x.dtype}, got {addend.dtype}")
    if addend.device != x.device:
        raise ValueError("addend must be on x's device")
    return _layer_norm(x, addend, weight, bias, eps)


def _layer_norm(x, addend, weight, bias, eps):
    if x.dim() < 1:
        raise ValueError("x must have at least one dimension")
    cols = x.shape[-1]
    if x.dtype not in SIXTEEN_BIT_DTYPES:
        raise ValueError(f"b200_layer_norm supports bfloat16 and float16, got {x.dtype}")
    if cols % 8 or cols > MAX_COLS or cols == 0:
        raise ValueError(f"b200_layer_norm needs a last dimension that is a multiple of 8 up to "
                         f"{MAX_COLS}, got {cols}")
    if not eps > 0:
        raise ValueError("eps must be positive")
    w = _vector(weight, cols, "weight", x)
    b = _vector(bias, cols, "bias", x)
    if torch.is_grad_enabled() and any(t is not None and t.requires_grad
                                       for t in (x, addend, weight, bias)):
        raise ValueError("b200_layer_norm is inference-only: it records no autograd graph")
    if not x.is_cuda:
        raise ValueError("b200_layer_norm runs on CUDA tensors only")
    y = torch.empty_like(x, memory_format=torch.contiguous_format)
    total = torch.empty_like(y) if addend is not None else None
    if y.numel() == 0:
        return total, y
    x2 = _rows(x, cols)
    y2 = y.view(-1, cols)
    a2 = _rows(addend, cols) if addend is not None else None
    s2 = total.view(-1, cols) if total is not None else None
    p = _native.LayerNormParams()
    _LN_LAYOUT.pack_into(p, 0, x2.data_ptr(), w.data_ptr() if w is not None else 0,
                         b.data_ptr() if b is not None else 0, y2.data_ptr(), x2.shape[0], cols,
                         x2.stride(0), y2.stride(0), float(eps), SIXTEEN_BIT_DTYPES[x.dtype],
                         a2.data_ptr() if a2 is not None else 0,
                         s2.data_ptr() if s2 is not None else 0,
                         a2.stride(0) if a2 is not None else 0,
                         s2.stride(0) if s2 is not None else 0)
    lib = _native.load_library()
    rc = lib.b200_layernorm_fwd(ctypes.byref(p),
                                ctypes.c_void_p(torch.cuda.current_stream(x.device).cuda_stream))
    if rc != _native.OK:
        raise_for_code("b200_layernorm_fwd", rc, x.device)
    return total, y
