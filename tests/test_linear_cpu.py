"""Host-side contract of ``b200_linear`` (no GPU needed): argument checks raise
before any device work, and the op never falls back to another implementation."""

import pytest
import torch

from b200_attention.linear import b200_linear, linear_supported


def test_cpu_tensors_are_rejected():
    x = torch.randn(4, 16, dtype=torch.bfloat16)
    w = torch.randn(8, 16, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        b200_linear(x, w)
    assert not linear_supported(x, w)


@pytest.mark.parametrize("kwargs,exc,match", [
    (dict(activation="relu"), ValueError, "activation"),
    (dict(masked_rows="keep"), ValueError, "masked_rows"),
    (dict(bias=torch.zeros(8, dtype=torch.float16)), TypeError, "bias"),
    (dict(residual=torch.zeros(4, 9, dtype=torch.bfloat16)), ValueError, "residual"),
    (dict(row_mask=torch.ones(4, dtype=torch.uint8)), TypeError, "row_mask"),
    (dict(row_mask=torch.ones(5, dtype=torch.bool)), ValueError, "row_mask"),
    (dict(row_mask=torch.ones(4, dtype=torch.bool), masked_rows="residual"), ValueError,
     "residual"),
])
def test_argument_errors(kwargs, exc, match):
    x = torch.randn(4, 16, dtype=torch.bfloat16)
    w = torch.randn(8, 16, dtype=torch.bfloat16)
    with pytest.raises(exc, match=match):
        b200_linear(x, w, **kwargs)


def test_shape_and_dtype_errors():
    w = torch.randn(8, 16, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="features"):
        b200_linear(torch.randn(4, 12, dtype=torch.bfloat16), w)
    with pytest.raises(ValueError, match="bfloat16 and float16"):
        b200_linear(torch.randn(4, 16), w.float())
    with pytest.raises(TypeError, match="weight"):
        b200_linear(torch.randn(4, 16, dtype=torch.bfloat16), w.half())
    with pytest.raises(ValueError, match="multiples of 8"):
        b200_linear(torch.randn(4, 12, dtype=torch.bfloat16), torch.randn(8, 12).bfloat16())


def test_autograd_is_refused():
    x = torch.randn(4, 16, dtype=torch.bfloat16)
    w = torch.randn(8, 16, dtype=torch.bfloat16, requires_grad=True)
    with pytest.raises(ValueError, match="inference-only"):
        b200_linear(x, w)
