"""GPU parity of the LayerNorm kernel against a plain PyTorch fp32 reference
(F.layer_norm on the fp32 values, rounded once to the element type).

The kernel's two-pass fp32 mean and variance differ from the reference's only
in the last bits, which can move a result across one rounding boundary:
|y - ref| <= 2^-7 |ref| + 2^-10 (bf16) and 2^-10 |ref| + 2^-13 (fp16), i.e.
one unit in the last place plus a small absolute slack near zero.
"""

import pytest
import torch
import torch.nn.functional as F

from b200_attention import read_device_errors
from b200_attention.layernorm import b200_layer_norm

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
TOL = {torch.bfloat16: (2.0**-7, 2.0**-10), torch.float16: (2.0**-10, 2.0**-13)}


def _check(shape, dtype=torch.bfloat16, affine=True, eps=1e-5, scale=1.0, shift=0.0, seed=0):
    g = torch.Generator("cpu").manual_seed(seed)
    cols = shape[-1]
    x = (torch.randn(*shape, generator=g) * scale + shift).to(dtype).to(DEV)
    w = (1 + 0.1 * torch.randn(cols, generator=g)).to(dtype).to(DEV) if affine else None
    b = (0.1 * torch.randn(cols, generator=g)).to(dtype).to(DEV) if affine else None
    y = b200_layer_norm(x, w, b, eps)
    ref = F.layer_norm(x.float(), (cols,), None if w is None else w.float(),
                       None if b is None else b.float(), eps).to(dtype)
    torch.cuda.synchronize()
    assert read_device_errors(DEV) == 0
    rtol, atol = TOL[dtype]
    diff = (y.float() - ref.float()).abs()
    assert bool((diff <= rtol * ref.float().abs() + atol).all()), diff.max().item()
    return y, ref


@pytest.mark.parametrize("shape", [(1, 8), (3, 24), (5, 264), (7, 1000), (16384, 1024), (2, 3, 4096),
                                   (33, 2048), (100, 520)])
def test_shapes(shape):
    _check(shape)


@pytest.mark.parametrize("kw", [dict(affine=False), dict(dtype=torch.float16),
                                dict(scale=30.0, shift=5.0), dict(shift=100.0, scale=0.5),
                                dict(shift=1000.0, scale=0.0), dict(eps=1e-2)],
                         ids=lambda kw: "-".join(f"{k}={v}" for k, v in kw.items()))
def test_variants(kw):
    _check((257, 1024), **kw)


def test_strided_input_and_module_semantics():
    ln = torch.nn.LayerNorm(1024).to(DEV, torch.bfloat16)
    with torch.no_grad():
        ln.weight.normal_(1.0, 0.1)
        ln.bias.normal_(0.0, 0.1)
    x = torch.randn(2048, 2048, device=DEV).to(torch.bfloat16)[:, ::2]  # non-contiguous rows
    y = b200_layer_norm(x, ln.weight.detach(), ln.bias.detach(), ln.eps)
    with torch.no_grad():
        ref = ln(x.contiguous())
    torch.cuda.synchronize()
    diff = (y.float() - ref.float()).abs()
    assert bool((diff <= 2.0**-6 * ref.float().abs() + 2.0**-9).all())


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", [(3, 24), (257, 1024), (2, 700, 1024), (33, 4096)])
def test_add_layer_norm(shape, dtype):
    """The residual sum is exactly torch's 16-bit add; the norm is that of the
    rounded sum (the reference normalises the stored 16-bit residual stream)."""
    from b200_attention.layernorm import b200_add_layer_norm

    g = torch.Generator("cpu").manual_seed(5)
    cols = shape[-1]
    x = torch.randn(*shape, generator=g).to(dtype).to(DEV)
    t = (0.5 * torch.randn(*shape, generator=g)).to(dtype).to(DEV)
    w = (1 + 0.1 * torch.randn(cols, generator=g)).to(dtype).to(DEV)
    b = (0.1 * torch.randn(cols, generator=g)).to(dtype).to(DEV)
    s, y = b200_add_layer_norm(x, t, w, b)
    s_ref = x + t
    ref = F.layer_norm(s_ref.float(), (cols,), w.float(), b.float(), 1e-5).to(dtype)
    torch.cuda.synchronize()
    assert torch.equal(s, s_ref)
    rtol, atol = TOL[dtype]
    diff = (y.float() - ref.float()).abs()
    assert bool((diff <= rtol * ref.float().abs() + atol).all()), diff.max().item()
