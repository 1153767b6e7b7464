"""C ABI checks that need no GPU: exports, struct layout, host-side validation.

The library must export every function ``include/b200_attn.h`` declares; the
ctypes mirror of ``b200_attn_fwd_params`` must match the C layout (compiled
here with gcc); ``b200_attn_check`` / ``b200_attn_query`` answer without any
CUDA call.
"""

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

from b200_attention import _native
from b200_attention.attention_dispatch import SM100_HEAD_DIMS
from b200_attention.build import LIB_PATH, build_native

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "b200_attn.h"


@pytest.fixture(scope="module")
def lib():
    build_native()  # no-op when the in-tree library is fresh
    return _native.load_library()


def declared_functions():
    text = HEADER.read_text()
    return re.findall(r"B200_ATTN_API\s+[\w\s\*]+?\b(b200_attn_\w+)\s*\(", text)


def test_header_declarations_are_mirrored():
    names = declared_functions()
    assert names, "no declarations parsed"
    assert set(names) == set(_native.EXPORTED_SYMBOLS)


def test_library_exports_every_declared_symbol(lib):
    out = subprocess.run(["nm", "-D", "--defined-only", str(LIB_PATH)], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r"\bT\s+(b200_attn_\w+)", out))
    for name in declared_functions():
        assert name in exported, name
        assert hasattr(lib, name)


def test_params_struct_layout_matches_c(tmp_path):
    fields = [f for f, _ in _native.FwdParams._fields_]
    src = tmp_path / "layout.c"
    body = "\n".join(f'  printf("{f} %zu\\n", offsetof(b200_attn_fwd_params, {f}));' for f in fields)
    src.write_text(f'#include <stdio.h>\n#include <stddef.h>\n#include "b200_attn.h"\n'
                   f'int main(void) {{\n  printf("size %zu\\n", sizeof(b200_attn_fwd_params));\n{body}\n  return 0;\n}}\n')
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c11", f"-I{ROOT / 'include'}", str(src), "-o", str(exe)], check=True)
    lines = dict(l.split() for l in subprocess.run([str(exe)], capture_output=True, text=True,
                                                   check=True).stdout.splitlines())
    assert int(lines["size"]) == ctypes.sizeof(_native.FwdParams)
    for f in fields:
        assert int(lines[f]) == getattr(_native.FwdParams, f).offset, f


def test_abi_version(lib):
    assert lib.b200_attn_abi_version() == 2


def test_launch_counter_starts_without_gpu_work(lib):
    assert lib.b200_attn_launch_count() >= 0


def test_query_agrees_with_planner_envelope(lib):
    """The C ABI and the planner agree on the head dims the kernel computes:
    every multiple of 8 up to 128."""
    from b200_attention.attention_dispatch import sm100_supports

    names = {_native.DTYPE_BF16: "bfloat16", _native.DTYPE_FP16: "float16",
             _native.DTYPE_FP32: "float32", 7: "float64"}
    for dtype, name in names.items():
        for d in (0, 4, 8, 12, 16, 32, 60, 64, 72, 96, 120, 128, 136, 256):
            supported = 1 if sm100_supports(name, d) else 0
            assert lib.b200_attn_query(dtype, d, 1, 0) == supported, (name, d)
    assert set(SM100_HEAD_DIMS) == set(range(8, 129, 8))
    assert lib.b200_attn_query(_native.DTYPE_FP32, 64, 1, 0) == 1
    assert lib.b200_attn_query(_native.DTYPE_FP32, 72, 1, 0) == 0


def test_launch_shape_agrees_with_planner(lib):
    """The planner's launch metadata and the kernel's own launch shape come
    from one definition: b200_attn_launch_shape reports what b200_attn_fwd
    launches, and the planner's constants must equal it."""
    from b200_attention.attention_dispatch import (SM100_BLOCK_M, SM100_BLOCK_N, SM100_NUM_WARPS,
                                                   _sm100_launch)

    names = {_native.DTYPE_BF16: "bfloat16", _native.DTYPE_FP16: "float16",
             _native.DTYPE_FP32: "float32"}
    for dtype, name in names.items():
        for d in SM100_HEAD_DIMS:
            shape = _native.launch_shape(dtype, d)
            if name == "float32" and d > 64:
                assert shape is None
                continue
            assert shape is not None, (dtype, d)
            launch = _sm100_launch(d, name)
            assert (shape["block_m"], shape["block_n"], shape["num_warps"], shape["ring_slots"]) == (
                launch.block_m, launch.block_n, launch.num_warps, launch.num_stages), (dtype, d)
            assert (shape["block_m"], shape["block_n"], shape["num_warps"]) == (
                SM100_BLOCK_M, SM100_BLOCK_N, SM100_NUM_WARPS)
            assert shape["rows_per_cta"] == 2 * shape["block_m"]
    assert _native.launch_shape(_native.DTYPE_BF16, 136) is None
    assert _native.launch_shape(9, 64) is None


def _params(**kw):
    p = _native.FwdParams()
    base = 0x10000
    p.q, p.k, p.v, p.o = base, base + 0x100000, base + 0x200000, base + 0x300000
    p.batch, p.heads, p.seq_len, p.head_dim = 2, 4, 256, 128
    st = (4 * 256 * 128, 256 * 128, 128)
    for name in ("q_stride", "k_stride", "v_stride", "o_stride"):
        getattr(p, name)[:] = st
    p.scale = 128 ** -0.5
    p.dtype = _native.DTYPE_BF16
    for k, v in kw.items():
        setattr(p, k, v)
    return p


def _check(lib, p):
    return lib.b200_attn_check(ctypes.byref(p))


def test_check_accepts_valid_params(lib):
    assert _check(lib, _params()) == _native.OK
    assert lib.b200_attn_launches_per_call(ctypes.byref(_params())) == 1
    # transposed projection view: [B,S,H,D] storage seen as [B,H,S,D]
    p = _params()
    for name in ("q_stride", "k_stride", "v_stride"):
        getattr(p, name)[:] = (256 * 4 * 128, 128, 4 * 128)
    assert _check(lib, p) == _native.OK


@pytest.mark.parametrize("kw,code", [
    (dict(q=None), _native.ERR_INVALID_ARGUMENT),
    (dict(batch=0), _native.ERR_INVALID_ARGUMENT),
    (dict(seq_len=0), _native.ERR_INVALID_ARGUMENT),
    (dict(scale=0.0), _native.ERR_INVALID_ARGUMENT),
    (dict(scale=-1.0), _native.ERR_INVALID_ARGUMENT),
    (dict(scale=float("inf")), _native.ERR_INVALID_ARGUMENT),
    (dict(dtype=5), _native.ERR_UNSUPPORTED),
    (dict(dtype=_native.DTYPE_FP32), _native.ERR_UNSUPPORTED),  # fp32 heads only up to 64
    (dict(head_dim=136), _native.ERR_UNSUPPORTED),
    (dict(head_dim=100), _native.ERR_UNSUPPORTED),
    (dict(q=0x10008), _native.ERR_ALIGNMENT),
    (dict(zero_masked_queries=1), _native.ERR_INVALID_ARGUMENT),
])
def test_check_rejects(lib, kw, code):
    assert _check(lib, _params(**kw)) == code


def test_check_accepts_fp32_up_to_head_dim_64(lib):
    p = _params(dtype=_native.DTYPE_FP32, head_dim=64)
    for name in ("q_stride", "k_stride", "v_stride", "o_stride"):
        getattr(p, name)[:] = (4 * 256 * 64, 256 * 64, 64)
    assert _check(lib, p) == _native.OK
    p.head_dim = 8  # 32-byte rows: 16-byte multiples for fp32
    for name in ("q_stride", "k_stride", "v_stride", "o_stride"):
        getattr(p, name)[:] = (4 * 256 * 8, 256 * 8, 8)
    assert _check(lib, p) == _native.OK
    getattr(p, "k_stride")[:] = (4 * 256 * 8, 256 * 8, 10)  # 40-byte rows
    assert _check(lib, p) == _native.ERR_ALIGNMENT


def test_check_rejects_unaligned_stride(lib):
    p = _params()
    p.k_stride[:] = (4 * 256 * 128, 256 * 128, 132)  # 264-byte rows: not a 16-byte multiple
    assert _check(lib, p) == _native.ERR_ALIGNMENT
    p = _params(seq_len=1)
    p.k_stride[:] = (4 * 1 * 128, 128, 3)  # seq stride irrelevant when S == 1
    assert _check(lib, p) == _native.OK


def test_error_strings(lib):
    for code in range(8):
        assert lib.b200_attn_error_string(code)
    assert b"unknown" in lib.b200_attn_error_string(99)


def test_packed_layout_fills_every_field_in_order():
    from b200_attention.fused_attention import _FWD_LAYOUT
    p = _native.FwdParams()
    ints = list(range(1, 26))  # 4 pointers, 4 sizes, 12 strides, mask pointer, 2 mask strides
    _FWD_LAYOUT.pack_into(p, 0, *ints[:23], 0.25, 26, 27, 28, 29)
    assert [p.q, p.k, p.v, p.o] == ints[:4]
    assert [p.batch, p.heads, p.seq_len, p.head_dim] == ints[4:8]
    assert list(p.q_stride) + list(p.k_stride) + list(p.v_stride) + list(p.o_stride) == ints[8:20]
    assert p.key_mask == 21 and list(p.mask_stride) == [22, 23]
    assert (p.scale, p.dtype, p.causal, p.zero_masked_queries, p.error_word) == (0.25, 26, 27, 28, 29)


def test_partial_entry_point_rejects_what_it_does_not_take(lib):
    """b200_attn_fwd_partial refuses key masks, zeroed queries and a missing or
    misaligned log-sum-exp buffer before touching the device."""
    def call(**kw):
        pp = _native.PartialParams()
        pp.base = _params()
        pp.lse = 0x20000
        pp.lse_stride[:] = (4 * 256, 256, 1)
        for key, val in kw.items():
            if key.startswith("base_"):
                setattr(pp.base, key[5:], val)
            else:
                setattr(pp, key, val)
        return lib.b200_attn_fwd_partial(ctypes.byref(pp), None)

    assert call(base_key_mask=0x30000) == _native.ERR_UNSUPPORTED
    assert call(base_zero_masked_queries=1) == _native.ERR_UNSUPPORTED
    assert call(lse=0) == _native.ERR_INVALID_ARGUMENT
    assert call(lse=0x20002) == _native.ERR_INVALID_ARGUMENT
    assert call(accumulate=2) == _native.ERR_INVALID_ARGUMENT
    assert call(reserved=1) == _native.ERR_INVALID_ARGUMENT
    assert lib.b200_attn_fwd_partial(None, None) == _native.ERR_INVALID_ARGUMENT


def test_partial_params_layout_matches_c(tmp_path):
    fields = [f for f, _ in _native.PartialParams._fields_]
    src = tmp_path / "layout.c"
    body = "\n".join(f'  printf("{f} %zu\\n", offsetof(b200_attn_partial_params, {f}));' for f in fields)
    src.write_text(f'#include <stdio.h>\n#include <stddef.h>\n#include "b200_attn.h"\n'
                   f'int main(void) {{\n  printf("size %zu\\n", sizeof(b200_attn_partial_params));\n{body}\n'
                   f'  return 0;\n}}\n')
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c11", f"-I{ROOT / 'include'}", str(src), "-o", str(exe)], check=True)
    lines = dict(l.split() for l in subprocess.run([str(exe)], capture_output=True, text=True,
                                                   check=True).stdout.splitlines())
    assert int(lines["size"]) == ctypes.sizeof(_native.PartialParams)
    for f in fields:
        assert int(lines[f]) == getattr(_native.PartialParams, f).offset, f
