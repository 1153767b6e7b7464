"""GPU parity of the fused linear kernel (``b200_linear``) against a plain
PyTorch fp32 reference of the same op.

The reference computes x @ W^T in fp32 (TF32 off) and applies the unfused
sequence's rounding points: the product plus bias rounded to the element type,
GELU in fp32 on that value and rounded again, the residual added in fp32 and
rounded once.  The kernel differs from it only by the fp32 summation order of
the product, which can move the rounded product t across one rounding
boundary; the tolerance is therefore two units in the last place of the
element type, taken at the larger of the result and t (a residual add can
cancel most of t):
|y - ref| <= 2^-6 (|ref| + |t|) + 2^-8 (bf16), 2^-9 (|ref| + |t|) + 2^-12 (fp16), and
the mean absolute error may not exceed 1.25x that of cuBLAS running the same
unfused sequence (F.linear, F.gelu, add, masked_fill) in the element type.
Rows whose mask is False must be exact: zeros, or the residual row unchanged.
"""

import pytest
import torch
import torch.nn.functional as F

from b200_attention import b200_linear, read_device_errors

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
TOL = {torch.bfloat16: (2.0**-6, 2.0**-8), torch.float16: (2.0**-9, 2.0**-12)}


def _reference(x, w, b, act, r, mask, mode):
    dt = x.dtype
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        t = x.float() @ w.float().T
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    if b is not None:
        t = t + b.float()
    t = t.to(dt).float()
    if act == "gelu":
        t = F.gelu(t).to(dt).float()
    y = (r.float() + t).to(dt) if r is not None else t.to(dt)
    if mask is not None:
        keep = mask[..., None]
        y = torch.where(keep, y, r if mode == "residual" else torch.zeros_like(y))
    return y, t


def _unfused(x, w, b, act, r, mask, mode):
    t = F.linear(x, w, b)
    if act == "gelu":
        t = F.gelu(t)
    if mask is not None and mode == "residual":
        t = t.masked_fill(~mask[..., None], 0)
    y = r + t if r is not None else t
    if mask is not None and mode == "zero":
        y = y.masked_fill(~mask[..., None], 0)
    return y


def _inputs(lead, n, k, dtype, bias, res, mask, seed):
    g = torch.Generator("cpu").manual_seed(seed)
    x = torch.randn(*lead, k, generator=g).to(dtype)
    w = (torch.randn(n, k, generator=g) * k**-0.5).to(dtype)
    b = (torch.randn(n, generator=g) * 0.1).to(dtype) if bias else None
    r = torch.randn(*lead, n, generator=g).to(dtype) if res else None
    m = (torch.rand(*lead, generator=g) > 0.3) if mask else None
    mv = lambda t: None if t is None else t.to(DEV)
    return mv(x), mv(w), mv(b), mv(r), mv(m)


def _check(lead, n, k, dtype=torch.bfloat16, act=None, bias=True, res=False, mask=False,
           mode="zero", seed=0):
    x, w, b, r, m = _inputs(lead, n, k, dtype, bias, res, mask, seed)
    y = b200_linear(x, w, b, activation=act, residual=r, row_mask=m, masked_rows=mode)
    ref, t = _reference(x, w, b, act, r, m, mode)
    base = _unfused(x, w, b, act, r, m, mode)
    torch.cuda.synchronize()
    assert read_device_errors(DEV) == 0
    assert y.shape == ref.shape and y.dtype == dtype
    rtol, atol = TOL[dtype]
    diff = (y.float() - ref.float()).abs()
    bound = rtol * (ref.float().abs() + t.abs()) + atol
    assert bool((diff <= bound).all()), f"max excess {(diff - bound).max().item():.3e}"
    base_mean = (base.float() - ref.float()).abs().mean().item()
    assert diff.mean().item() <= 1.25 * base_mean + 1e-6
    if m is not None:
        off = ~m
        expect = r[off] if mode == "residual" else torch.zeros_like(y[off])
        assert torch.equal(y[off], expect)
    return y


# (lead dims, N, K): one-CTA kernel (M <= 128 or N <= 128) and CTA-pair kernel,
# with tails in every dimension
SHAPES = [((1,), 8, 8), ((7,), 24, 40), ((128,), 128, 64), ((129,), 136, 72),
          ((300,), 264, 520), ((257,), 256, 64), ((384,), 520, 136), ((1000,), 1024, 1024),
          ((2048,), 3072, 1024), ((2, 700), 1024, 512), ((256,), 1024, 4096)]


@pytest.mark.parametrize("lead,n,k", SHAPES)
def test_plain_shapes(lead, n, k):
    _check(lead, n, k)


@pytest.mark.parametrize("kw", [
    dict(act="gelu"),
    dict(res=True),
    dict(res=True, mask=True, mode="residual"),
    dict(res=True, mask=True, mode="zero"),
    dict(mask=True),
    dict(bias=False),
    dict(act="gelu", res=True, mask=True),
    dict(dtype=torch.float16),
    dict(dtype=torch.float16, act="gelu", res=True, mask=True, mode="residual"),
], ids=lambda kw: "-".join(f"{k}={v}" for k, v in kw.items()))
@pytest.mark.parametrize("lead,n,k", [((1000,), 1024, 1024), ((333,), 264, 200), ((96,), 64, 48)])
def test_epilogues(lead, n, k, kw):
    _check(lead, n, k, **kw)


def test_decoder_shapes_with_mask():
    """The decoder's four projections at B=2, S=2048, d=1024, FFN 4096, with a
    padded batch (rows past each sequence's length masked)."""
    lead = (2, 2048)
    _check(lead, 3072, 1024)
    _check(lead, 1024, 1024, res=True, mask=True, mode="residual", seed=1)
    _check(lead, 4096, 1024, act="gelu", seed=2)
    _check(lead, 1024, 4096, res=True, mask=True, mode="zero", seed=3)


def test_strided_inputs_and_repeat_calls():
    x, w, b, r, _ = _inputs((512,), 256, 512, torch.bfloat16, True, True, False, 5)
    xt = x.t().contiguous().t()  # column-major storage: copied to rows internally
    y1 = b200_linear(xt, w, b, residual=r)
    y2 = b200_linear(x, w, b, residual=r)
    torch.cuda.synchronize()
    assert torch.equal(y1, y2)
    assert read_device_errors(DEV) == 0


def test_graph_capture_replays_identically():
    x, w, b, _, _ = _inputs((1024,), 1024, 1024, torch.bfloat16, True, False, False, 6)
    eager = b200_linear(x, w, b, activation="gelu")
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        b200_linear(x, w, b, activation="gelu")  # warm-up outside capture
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = b200_linear(x, w, b, activation="gelu")
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)
    assert read_device_errors(DEV) == 0
