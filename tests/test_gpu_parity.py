"""GPU parity of the sm_100a kernel against the CPU oracle (reference op order).

Inputs follow the reference's generator (seeded torch.randn, fp32, cast to the
model dtype).  Small shapes are checked against the CPU oracle; edge cases
mirror the reference's tests: partial tiles, a single token, padded keys,
BSHD output equal to BHSD (test/test_triton_fused_attention.py:760-817).
"""

import pytest
import torch

from b200_attention import b200_fused_attention, read_device_errors
from oracle.reference_attention import reference_attention, zero_masked_rows
from parity import assert_close, prefix_mask, seeded_qkv

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def _run(shape, dtype, causal, lengths=None, seed=1234, zero_q=False, bshd=False):
    B, H, S, D = shape
    q, k, v = seeded_qkv(shape, dtype, seed)
    mask = prefix_mask(B, S, lengths) if lengths is not None else None
    ref = reference_attention(q, k, v, mask, causal, D**-0.5)
    if zero_q:
        ref = zero_masked_rows(ref, mask)
    out = b200_fused_attention(
        q.to(DEV), k.to(DEV), v.to(DEV),
        None if mask is None else mask.to(DEV),
        causal, output_bshd=bshd, zero_masked_queries=zero_q,
    )
    torch.cuda.synchronize()
    assert read_device_errors(DEV) == 0
    if bshd:
        out = out.transpose(1, 2)
    return out, ref


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("S", [128, 256, 512])
@pytest.mark.parametrize("causal", [False, True])
def test_aligned_shapes(D, S, causal):
    out, ref = _run((1, 2, S, D), torch.bfloat16, causal)
    assert_close(out, ref, f"D={D} S={S} causal={causal}")


@pytest.mark.parametrize("S", [1, 33, 97, 129, 200, 257, 300])
@pytest.mark.parametrize("causal", [False, True])
def test_partial_tiles(S, causal):
    out, ref = _run((2, 2, S, 128), torch.bfloat16, causal, seed=7)
    assert_close(out, ref, f"S={S} causal={causal}")


@pytest.mark.parametrize("causal", [False, True])
def test_fp16(causal):
    out, ref = _run((1, 2, 384, 64), torch.float16, causal, seed=11)
    assert_close(out, ref, "fp16")


@pytest.mark.parametrize("causal", [False, True])
def test_key_padding_mask(causal):
    out, ref = _run((3, 2, 520, 128), torch.bfloat16, causal, lengths=[520, 300, 77], seed=5)
    assert_close(out, ref, "mask")


def test_zero_masked_queries():
    out, ref = _run((2, 2, 700, 128), torch.bfloat16, False, lengths=[650, 129], seed=3, zero_q=True)
    assert_close(out, ref, "zero_q")


def test_bshd_equals_bhsd():
    q, k, v = (t.to(DEV) for t in seeded_qkv((2, 3, 300, 128), torch.bfloat16, 9))
    a = b200_fused_attention(q, k, v, None, True)
    b = b200_fused_attention(q, k, v, None, True, output_bshd=True)
    assert torch.equal(a, b.transpose(1, 2))


def test_transposed_projection_views():
    """q/k/v as [B,S,H,D] projections viewed [B,H,S,D] (reference adapter :2287-2292)."""
    B, S, H, D = 2, 333, 4, 64
    gen = torch.Generator("cpu").manual_seed(21)
    x = torch.randn((3, B, S, H * D), generator=gen).to(torch.bfloat16)
    q, k, v = (t.view(B, S, H, D).transpose(1, 2) for t in x)
    ref = reference_attention(q, k, v, None, True, D**-0.5)
    out = b200_fused_attention(q.to(DEV), k.to(DEV), v.to(DEV), None, True)
    torch.cuda.synchronize()
    assert_close(out, ref, "views")


def test_fully_masked_rows_are_nan():
    """All keys of batch 1 masked: torch.softmax gives NaN rows; so must the kernel."""
    out, ref = _run((2, 1, 130, 128), torch.bfloat16, False, lengths=[130, 0], seed=2)
    assert torch.isnan(out[1].float()).all() and torch.isnan(ref[1].float()).all()
    assert_close(out, ref, "nan rows")


@pytest.mark.parametrize("D", [8, 16, 24, 32, 40, 72, 96, 120])
@pytest.mark.parametrize("causal", [False, True])
def test_narrow_head_dims(D, causal):
    """Head dims other than 64 and 128 run the 64- or 128-wide instance, whose
    TMA boxes read the missing columns as zeros and whose output store clips
    them; the result must equal attention at the true head dim."""
    out, ref = _run((2, 3, 300, D), torch.bfloat16, causal, lengths=[300, 123])
    assert out.shape == ref.shape
    assert_close(out, ref, f"D={D}")


def test_narrow_head_dim_bshd_and_out():
    q, k, v = seeded_qkv((2, 4, 128, 32), torch.bfloat16, 77)
    ref = reference_attention(q, k, v, None, True, 32 ** -0.5)
    out = torch.empty((2, 128, 4, 32), device=DEV, dtype=torch.bfloat16)
    res = b200_fused_attention(q.to(DEV), k.to(DEV), v.to(DEV), None, True, output_bshd=True,
                               out=out)
    torch.cuda.synchronize()
    assert res is out and out.is_contiguous()
    assert_close(out.transpose(1, 2), ref, "D=32 BSHD")


@pytest.mark.parametrize("D", [64, 128])
def test_zero_masked_queries_causal(D):
    out, ref = _run((3, 2, 600, D), torch.bfloat16, True, lengths=[600, 257, 1], seed=13, zero_q=True)
    assert_close(out, ref, "zero_q causal")


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("D,dtype", [(64, torch.float16), (128, torch.bfloat16)])
def test_arbitrary_key_masks(causal, D, dtype):
    """Masks with holes (not a valid-length prefix), as the operator accepts any
    boolean [B, S] key mask; rows that see no valid key are NaN like the reference."""
    B, H, S = 2, 2, 389
    q, k, v = seeded_qkv((B, H, S, D), dtype, 17)
    gen = torch.Generator("cpu").manual_seed(99)
    mask = torch.rand((B, S), generator=gen) < 0.6
    mask[1, :5] = False  # early causal rows of batch 1 see no valid key -> NaN
    ref = reference_attention(q, k, v, mask, causal, D ** -0.5)
    out = b200_fused_attention(q.to(DEV), k.to(DEV), v.to(DEV), mask.to(DEV), causal)
    torch.cuda.synchronize()
    assert read_device_errors(DEV) == 0
    assert_close(out, ref, "holes")


def test_strided_mask_view():
    """A mask that is a strided view (seq stride 2) goes through the scalar path."""
    B, H, S, D = 2, 2, 300, 128
    q, k, v = seeded_qkv((B, H, S, D), torch.bfloat16, 23)
    wide = torch.zeros((B, 2 * S), dtype=torch.bool)
    wide[0, 0:2 * 250:2] = True
    wide[1, 0:2 * 77:2] = True
    mask = wide[:, ::2]
    assert mask.stride(1) == 2
    ref = reference_attention(q, k, v, mask.contiguous(), False, D ** -0.5)
    out = b200_fused_attention(q.to(DEV), k.to(DEV), v.to(DEV), wide.to(DEV)[:, ::2], False)
    torch.cuda.synchronize()
    assert_close(out, ref, "strided mask")


def test_contract_errors_raise_not_crash():
    """Contract violations come back as exceptions from the host-side checks;
    nothing is launched."""
    base = torch.zeros((1, 1, 64, 136), device=DEV, dtype=torch.bfloat16)
    q = base[..., 1:129]  # 2-byte offset: not 16-byte aligned for TMA
    ok = torch.zeros((1, 1, 64, 128), device=DEV, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        b200_fused_attention(q, ok, ok, None, True)
    with pytest.raises(ValueError):
        b200_fused_attention(ok, ok, ok, None, True, scale=-1.0)
    with pytest.raises(ValueError):
        b200_fused_attention(ok.float(), ok.float(), ok.float(), None, True)
    with pytest.raises(ValueError):
        b200_fused_attention(ok, ok, ok, None, True, zero_masked_queries=True)
    with pytest.raises(TypeError):
        b200_fused_attention(ok, ok, ok, torch.ones((1, 64), device=DEV), True)
    assert read_device_errors(DEV) == 0


def test_fp16_reference_published_shape():
    """The reference's only published attention timing: fp16 B64 H4 S1024 D32
    causal (its two-pass Triton path, model/triton_fused_attention.py:1728-1837,
    docs/TECH_REPORT.md:98-111).  The kernel runs the whole batch; the oracle
    checks eight batch entries spread over it, all heads."""
    B, H, S, D = 64, 4, 1024, 32
    q, k, v = seeded_qkv((B, H, S, D), torch.float16, 1234)
    out = b200_fused_attention(q.to(DEV), k.to(DEV), v.to(DEV), None, True).cpu()
    torch.cuda.synchronize()
    assert read_device_errors(DEV) == 0
    for b in (0, 9, 18, 27, 36, 45, 54, 63):
        ref = reference_attention(q[b:b + 1], k[b:b + 1], v[b:b + 1], None, True, D ** -0.5)
        assert_close(out[b:b + 1], ref, f"tr batch {b}")


@pytest.mark.parametrize("causal", [False, True])
def test_fp16_head_dim_128_masked(causal):
    out, ref = _run((2, 2, 1100, 128), torch.float16, causal, lengths=[1100, 500], seed=41)
    assert_close(out, ref, f"fp16 D=128 causal={causal}")


def test_fp16_long_causal_head_dim_64():
    out, ref = _run((1, 4, 2048, 64), torch.float16, True, seed=43)
    assert_close(out, ref, "fp16 S=2048 D=64")


@pytest.mark.parametrize("D", [8, 24, 40, 96])
@pytest.mark.parametrize("causal", [False, True])
def test_fp16_narrow_head_dims(D, causal):
    out, ref = _run((2, 3, 300, D), torch.float16, causal, lengths=[300, 123], seed=47)
    assert_close(out, ref, f"fp16 D={D}")


def test_fp16_zero_masked_queries_bshd():
    out, ref = _run((2, 2, 640, 128), torch.float16, True, lengths=[640, 200], seed=53, zero_q=True,
                    bshd=True)
    assert_close(out, ref, "fp16 zero_q bshd")



# fp32 inputs: the fp32 instance multiplies on the tensor cores as TF32 (the
# precision of the reference's fp32 tiled kernel, model/triton_fused_attention.py:
# 235-356) with an fp32 softmax and fp32 output; the oracle is exact fp32
# attention in the reference's operation order, and the bound is the same
# max-abs <= 2e-2 / mean-abs <= 2e-3 as for the 16-bit types.


def test_fp32_cfg1_full():
    """B2 H8 S512 D64 causal in fp32 (the reference's CPU dtype)."""
    out, ref = _run((2, 8, 512, 64), torch.float32, True)
    assert out.dtype == torch.float32
    assert_close(out, ref, "fp32 cfg1")


@pytest.mark.parametrize("D", [8, 16, 32, 64])
@pytest.mark.parametrize("causal", [False, True])
def test_fp32_head_dims(D, causal):
    out, ref = _run((2, 3, 300, D), torch.float32, causal, lengths=[300, 123], seed=61)
    assert_close(out, ref, f"fp32 D={D}")


@pytest.mark.parametrize("S", [1, 33, 128, 129, 257])
def test_fp32_partial_tiles(S):
    out, ref = _run((2, 2, S, 64), torch.float32, True, seed=67)
    assert_close(out, ref, f"fp32 S={S}")


def test_fp32_small_head_full_row():
    """The reference's fp32 D=8 small-head case (S <= 128, its Gluon kernel,
    model/triton_gluon_attention.py:184-317): B4 H16 S128 D8."""
    out, ref = _run((4, 16, 128, 8), torch.float32, True, seed=71)
    assert_close(out, ref, "fp32 D=8 S=128")


def test_fp32_long_causal():
    """The reference's fp32 tiled envelope (causal, S >= 1024, D 32/64)."""
    for D in (32, 64):
        out, ref = _run((1, 4, 2048, D), torch.float32, True, seed=73)
        assert_close(out, ref, f"fp32 S=2048 D={D}")


def test_fp32_masks_nan_rows_zero_queries_and_bshd():
    out, ref = _run((2, 1, 130, 64), torch.float32, False, lengths=[130, 0], seed=79)
    assert torch.isnan(out[1]).all() and torch.isnan(ref[1]).all()
    assert_close(out, ref, "fp32 nan rows")
    out, ref = _run((3, 2, 600, 64), torch.float32, True, lengths=[600, 257, 1], seed=83,
                    zero_q=True, bshd=True)
    assert_close(out, ref, "fp32 zero_q bshd")


def test_fp32_head_dim_above_64_is_refused():
    ok = torch.zeros((1, 1, 64, 128), device=DEV, dtype=torch.float32)
    with pytest.raises(ValueError, match="float32"):
        b200_fused_attention(ok, ok, ok, None, True)
