"""C ABI and host-side contract of the LayerNorm kernel (no GPU needed)."""

import ctypes
import re
import subprocess
from pathlib import Path

import pytest
import torch

from b200_attention import _native
from b200_attention.build import LIB_PATH, build_native
from b200_attention.layernorm import b200_layer_norm, layer_norm_supported

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "b200_layernorm.h"


@pytest.fixture(scope="module")
def lib():
    build_native()
    return _native.load_library()


def test_header_declarations_are_mirrored_and_exported(lib):
    names = re.findall(r"B200_ATTN_API\s+[\w\s\*]+?\b(b200_layernorm_\w+)\s*\(", HEADER.read_text())
    assert set(names) == set(_native.LAYERNORM_SYMBOLS)
    out = subprocess.run(["nm", "-D", "--defined-only", str(LIB_PATH)], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r"\bT\s+(b200_layernorm_\w+)", out))
    assert set(names) <= exported


def test_params_struct_layout_matches_c(tmp_path):
    fields = [f for f, _ in _native.LayerNormParams._fields_]
    src = tmp_path / "layout.c"
    body = "\n".join(f'  printf("{f} %zu\\n", offsetof(b200_layernorm_params, {f}));' for f in fields)
    src.write_text(f'#include <stdio.h>\n#include <stddef.h>\n#include "b200_layernorm.h"\n'
                   f'int main(void) {{\n  printf("size %zu\\n", sizeof(b200_layernorm_params));\n'
                   f'{body}\n  return 0;\n}}\n')
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c11", f"-I{ROOT / 'include'}", str(src), "-o", str(exe)], check=True)
    lines = dict(l.split() for l in subprocess.run([str(exe)], capture_output=True, text=True,
                                                   check=True).stdout.splitlines())
    assert int(lines["size"]) == ctypes.sizeof(_native.LayerNormParams)
    for f in fields:
        assert int(lines[f]) == getattr(_native.LayerNormParams, f).offset, f


def _params(**kw):
    p = _native.LayerNormParams()
    # operands 256 MB apart: no two ranges overlap unless a case says so
    p.x, p.y, p.weight, p.bias = 0x10000000, 0x20000000, 0x30000000, 0x30000800
    p.rows, p.cols, p.x_row_stride, p.y_row_stride = 16384, 1024, 1024, 1024
    p.eps, p.dtype = 1e-5, _native.DTYPE_BF16
    for k, v in kw.items():
        setattr(p, k, v)
    return p


@pytest.mark.parametrize("kw,code", [
    ({}, _native.OK),
    (dict(weight=None, bias=None), _native.OK),
    (dict(rows=1, x_row_stride=0), _native.OK),
    (dict(x=None), _native.ERR_INVALID_ARGUMENT),
    (dict(rows=0), _native.ERR_INVALID_ARGUMENT),
    (dict(rows=8 * 0x7fffffff + 1), _native.ERR_INVALID_ARGUMENT),
    (dict(eps=0.0), _native.ERR_INVALID_ARGUMENT),
    (dict(eps=float("nan")), _native.ERR_INVALID_ARGUMENT),
    (dict(dtype=3), _native.ERR_UNSUPPORTED),
    (dict(cols=8192, x_row_stride=8192, y_row_stride=8192), _native.ERR_UNSUPPORTED),
    (dict(cols=1020, x_row_stride=1024, y_row_stride=1024), _native.ERR_ALIGNMENT),
    (dict(x_row_stride=1000), _native.ERR_INVALID_ARGUMENT),
    (dict(y=0x20000004), _native.ERR_ALIGNMENT),
    (dict(bias=0x30000802), _native.ERR_ALIGNMENT),
    (dict(addend=0x40000000, addend_row_stride=1024), _native.OK),
    (dict(addend=0x40000000, addend_row_stride=1024, sum=0x10000000, sum_row_stride=1024),
     _native.OK),  # the sum written over x in place
    (dict(sum=0x50000000, sum_row_stride=1024), _native.ERR_INVALID_ARGUMENT),  # sum without addend
    (dict(addend=0x40000000, addend_row_stride=1024, sum=0x20000000, sum_row_stride=1024),
     _native.ERR_INVALID_ARGUMENT),  # sum onto the normalised output
    (dict(addend=0x40000000, addend_row_stride=1000), _native.ERR_INVALID_ARGUMENT),
    (dict(addend=0x40000008, addend_row_stride=1024), _native.ERR_ALIGNMENT),
    # in place (an output that IS an input) is allowed; any other overlap is not
    (dict(y=0x10000000), _native.OK),
    (dict(y=0x10000010), _native.ERR_INVALID_ARGUMENT),  # y shifted over x by 8 elements
    (dict(y=0x10000000, y_row_stride=2048), _native.ERR_INVALID_ARGUMENT),  # same base, other stride
    (dict(y=0x0ffff000), _native.ERR_INVALID_ARGUMENT),  # y's last rows over x's first
    (dict(addend=0x40000000, addend_row_stride=1024, y=0x40000000), _native.OK),
    (dict(addend=0x40000000, addend_row_stride=1024, sum=0x40000800, sum_row_stride=1024),
     _native.ERR_INVALID_ARGUMENT),  # sum shifted over the addend
    (dict(addend=0x40000000, addend_row_stride=1024, sum=0x1fffff00, sum_row_stride=1024),
     _native.ERR_INVALID_ARGUMENT),  # sum's last row over y's first
])
def test_check(lib, kw, code):
    assert lib.b200_layernorm_check(ctypes.byref(_params(**kw))) == code


def test_python_argument_errors():
    x = torch.randn(4, 64, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        b200_layer_norm(x)
    assert not layer_norm_supported(x, None)
    with pytest.raises(ValueError, match="multiple of 8"):
        b200_layer_norm(torch.randn(4, 60, dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="bfloat16 and float16"):
        b200_layer_norm(torch.randn(4, 64))
    with pytest.raises(TypeError, match="weight"):
        b200_layer_norm(x, torch.ones(64))
    with pytest.raises(ValueError, match="shape"):
        b200_layer_norm(x, torch.ones(32, dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="eps"):
        b200_layer_norm(x, eps=0.0)
    with pytest.raises(ValueError, match="inference-only"):
        b200_layer_norm(x, torch.ones(64, dtype=torch.bfloat16, requires_grad=True))


def test_packed_layout_fills_every_field_in_order():
    from b200_attention.layernorm import _LN_LAYOUT
    p = _native.LayerNormParams()
    values = [1, 2, 3, 4, 5, 6, 7, 8, 0.5, 9, 10, 11, 12, 13]
    _LN_LAYOUT.pack_into(p, 0, *values)
    assert [getattr(p, f) for f, _ in _native.LayerNormParams._fields_] == values
