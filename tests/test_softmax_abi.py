"""C ABI and host-side contract of the row-softmax kernel (no GPU needed)."""

import ctypes
import re
import subprocess
from pathlib import Path

import pytest
import torch

from b200_attention import _native
from b200_attention.build import LIB_PATH, build_native
from b200_attention.softmax import _SOFTMAX_LAYOUT, b200_attention_softmax, triton_attention_softmax

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "b200_softmax.h"


@pytest.fixture(scope="module")
def lib():
    build_native()
    return _native.load_library()


def test_header_declarations_are_mirrored_and_exported(lib):
    names = re.findall(r"B200_ATTN_API\s+[\w\s\*]+?\b(b200_softmax_\w+)\s*\(", HEADER.read_text())
    assert set(names) == set(_native.SOFTMAX_SYMBOLS)
    out = subprocess.run(["nm", "-D", "--defined-only", str(LIB_PATH)], capture_output=True,
                         text=True, check=True).stdout
    assert set(names) <= set(re.findall(r"\bT\s+(b200_softmax_\w+)", out))


def test_params_struct_layout_matches_c(tmp_path):
    fields = [f for f, _ in _native.SoftmaxParams._fields_]
    src = tmp_path / "layout.c"
    body = "\n".join(f'  printf("{f} %zu\\n", offsetof(b200_softmax_params, {f}));' for f in fields)
    src.write_text(f'#include <stdio.h>\n#include <stddef.h>\n#include "b200_softmax.h"\n'
                   f'int main(void) {{\n  printf("size %zu\\n", sizeof(b200_softmax_params));\n'
                   f'  printf("max %d\\n", B200_SOFTMAX_MAX_SEQ);\n{body}\n  return 0;\n}}\n')
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c11", f"-I{ROOT / 'include'}", str(src), "-o", str(exe)], check=True)
    lines = dict(l.split() for l in subprocess.run([str(exe)], capture_output=True, text=True,
                                                   check=True).stdout.splitlines())
    assert int(lines["size"]) == ctypes.sizeof(_native.SoftmaxParams) == _SOFTMAX_LAYOUT.size
    assert int(lines["max"]) == _native.SOFTMAX_MAX_SEQ
    for f in fields:
        assert int(lines[f]) == getattr(_native.SoftmaxParams, f).offset, f


def _params(**kw):
    p = _native.SoftmaxParams()
    p.scores, p.probs = 0x10000000, 0x1000000000  # 64 GB apart: disjoint for every case
    p.batch, p.heads, p.seq_len = 8, 16, 1024
    p.scale, p.dtype = 0.125, _native.DTYPE_BF16
    for k, v in kw.items():
        setattr(p, k, v)
    return p


@pytest.mark.parametrize("kw,code", [
    ({}, _native.OK),
    (dict(probs=0x10000000), _native.OK),  # in place
    (dict(dtype=_native.DTYPE_FP32), _native.OK),
    (dict(dtype=_native.DTYPE_FP16, seq_len=33), _native.OK),
    (dict(seq_len=65536, batch=1, heads=1), _native.OK),
    (dict(seq_len=65537, batch=1, heads=1), _native.ERR_INVALID_ARGUMENT),
    (dict(scores=None), _native.ERR_INVALID_ARGUMENT),
    (dict(batch=0), _native.ERR_INVALID_ARGUMENT),
    (dict(scale=0.0), _native.ERR_INVALID_ARGUMENT),
    (dict(scale=float("nan")), _native.ERR_INVALID_ARGUMENT),
    (dict(reserved=1), _native.ERR_INVALID_ARGUMENT),
    (dict(dtype=7), _native.ERR_UNSUPPORTED),
    (dict(scores=0x10000001), _native.ERR_ALIGNMENT),
    (dict(dtype=_native.DTYPE_FP32, probs=0x1000000002), _native.ERR_ALIGNMENT),
    (dict(probs=0x10000010), _native.ERR_INVALID_ARGUMENT),  # shifted over the scores
    (dict(probs=0x0ffffff0), _native.ERR_INVALID_ARGUMENT),
])
def test_check(lib, kw, code):
    assert lib.b200_softmax_check(ctypes.byref(_params(**kw))) == code


def test_python_contract_matches_the_reference_seam():
    """Same checks and exception types as triton_attention_softmax
    (model/triton_softmax.py:106-140)."""
    assert triton_attention_softmax is b200_attention_softmax
    x = torch.randn(1, 2, 8, 8)
    with pytest.raises(ValueError, match="shape"):
        b200_attention_softmax(x[0], None, 0.5, False)
    with pytest.raises(ValueError, match="square"):
        b200_attention_softmax(torch.randn(1, 2, 8, 4), None, 0.5, False)
    with pytest.raises(ValueError, match="CUDA"):
        b200_attention_softmax(x, None, 0.5, False)


def test_packed_layout_fills_every_field_in_order():
    p = _native.SoftmaxParams()
    values = [1, 2, 3, 4, 5, 6, 7, 8, 0.5, 9, 10, 11]
    _SOFTMAX_LAYOUT.pack_into(p, 0, *values)
    got = [getattr(p, f) for f, _ in _native.SoftmaxParams._fields_]
    got = got[:6] + list(got[6]) + got[7:]
    assert got == values
