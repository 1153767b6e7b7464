"""C ABI of the fused linear layer (``include/b200_linear.h``), checked without a GPU.

The library exports every function the header declares, the ctypes mirror of
``b200_linear_params`` matches the C layout (compiled here with gcc), and
``b200_linear_check`` / ``b200_linear_tile_n`` answer without any CUDA call.
"""

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

from b200_attention import _native
from b200_attention.build import LIB_PATH, build_native

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "b200_linear.h"


@pytest.fixture(scope="module")
def lib():
    build_native()
    return _native.load_library()


def declared_functions():
    text = HEADER.read_text()
    return re.findall(r"B200_ATTN_API\s+[\w\s\*]+?\b(b200_linear_\w+)\s*\(", text)


def test_header_declarations_are_mirrored():
    names = declared_functions()
    assert names
    assert set(names) == set(_native.LINEAR_SYMBOLS)


def test_library_exports_every_declared_symbol(lib):
    out = subprocess.run(["nm", "-D", "--defined-only", str(LIB_PATH)], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r"\bT\s+(b200_linear_\w+)", out))
    for name in declared_functions():
        assert name in exported, name
        assert hasattr(lib, name)


def test_params_struct_layout_matches_c(tmp_path):
    fields = [f for f, _ in _native.LinearParams._fields_]
    src = tmp_path / "layout.c"
    body = "\n".join(f'  printf("{f} %zu\\n", offsetof(b200_linear_params, {f}));' for f in fields)
    src.write_text(f'#include <stdio.h>\n#include <stddef.h>\n#include "b200_linear.h"\n'
                   f'int main(void) {{\n  printf("size %zu\\n", sizeof(b200_linear_params));\n'
                   f'{body}\n  return 0;\n}}\n')
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c11", f"-I{ROOT / 'include'}", str(src), "-o", str(exe)], check=True)
    lines = dict(l.split() for l in subprocess.run([str(exe)], capture_output=True, text=True,
                                                   check=True).stdout.splitlines())
    assert int(lines["size"]) == ctypes.sizeof(_native.LinearParams)
    for f in fields:
        assert int(lines[f]) == getattr(_native.LinearParams, f).offset, f


def _params(**kw):
    p = _native.LinearParams()
    # operands 256 MB apart: no two ranges overlap
    p.x, p.w, p.y = 0x10000000, 0x20000000, 0x30000000
    p.bias = 0x40000000
    p.m, p.n, p.k = 16384, 4096, 1024
    p.x_row_stride, p.w_row_stride, p.y_row_stride = 1024, 1024, 4096
    p.dtype = _native.DTYPE_BF16
    for key, value in kw.items():
        setattr(p, key, value)
    return p


def _check(lib, p):
    return lib.b200_linear_check(ctypes.byref(p))


def test_check_accepts_valid_params(lib):
    assert _check(lib, _params()) == _native.OK
    assert _check(lib, _params(activation=_native.LINEAR_ACT_GELU)) == _native.OK
    res = 0x50000000
    assert _check(lib, _params(residual=res, residual_row_stride=4096, row_mask=0x7000,
                               masked_rows=_native.LINEAR_MASKED_KEEP_RESIDUAL)) == _native.OK
    assert _check(lib, _params(m=1, x_row_stride=3)) == _native.OK  # row stride unused for one row
    assert _check(lib, _params(bias=None, dtype=_native.DTYPE_FP16)) == _native.OK


@pytest.mark.parametrize("kw,code", [
    (dict(x=None), _native.ERR_INVALID_ARGUMENT),
    (dict(y=None), _native.ERR_INVALID_ARGUMENT),
    (dict(m=0), _native.ERR_INVALID_ARGUMENT),
    (dict(k=0), _native.ERR_INVALID_ARGUMENT),
    (dict(n=1 << 31), _native.ERR_INVALID_ARGUMENT),
    (dict(dtype=5), _native.ERR_UNSUPPORTED),
    (dict(activation=2), _native.ERR_INVALID_ARGUMENT),
    (dict(masked_rows=2), _native.ERR_INVALID_ARGUMENT),
    (dict(reserved=1), _native.ERR_INVALID_ARGUMENT),
    (dict(row_mask=0x7000, masked_rows=1), _native.ERR_INVALID_ARGUMENT),  # keep needs residual
    (dict(x_row_stride=1000), _native.ERR_INVALID_ARGUMENT),  # shorter than K
    (dict(n=4100, y_row_stride=4100, k=1024), _native.ERR_ALIGNMENT),  # N not a multiple of 8
    (dict(k=1020, x_row_stride=1024, w_row_stride=1024), _native.ERR_ALIGNMENT),
    (dict(x=0x10000008), _native.ERR_ALIGNMENT),
    (dict(bias=0x40000002), _native.ERR_ALIGNMENT),
    (dict(y_row_stride=4100), _native.ERR_ALIGNMENT),
    # y overlapping an input: its stores would race the input's loads
    (dict(y=0x10000000), _native.ERR_INVALID_ARGUMENT),  # y == x
    (dict(y=0x1ffff000), _native.ERR_INVALID_ARGUMENT),  # y's first rows over W
    (dict(bias=0x30000100), _native.ERR_INVALID_ARGUMENT),
    (dict(residual=0x30000000, residual_row_stride=4096), _native.ERR_INVALID_ARGUMENT),
    (dict(residual=0x2ffff000, residual_row_stride=4096), _native.ERR_INVALID_ARGUMENT),
    (dict(row_mask=0x30000010), _native.ERR_INVALID_ARGUMENT),
])
def test_check_rejects(lib, kw, code):
    assert _check(lib, _params(**kw)) == code


def test_tile_width(lib):
    assert lib.b200_linear_tile_n(ctypes.byref(_params()), 148) == 256
    assert lib.b200_linear_tile_n(ctypes.byref(_params(n=128, y_row_stride=128)), 148) == 128
    assert lib.b200_linear_tile_n(ctypes.byref(_params(m=0)), 148) == 0


def test_packed_layout_fills_every_field_in_order():
    from b200_attention.linear import _LINEAR_LAYOUT
    p = _native.LinearParams()
    values = list(range(1, 19))
    _LINEAR_LAYOUT.pack_into(p, 0, *values)
    got = [getattr(p, f) for f, _ in _native.LinearParams._fields_]
    assert got == values
