"""Build the sm_100a attention library in-tree with nvcc.

The shared library is torch-free: it exports the C ABI declared in
``include/b200_attn.h``, ``include/b200_linear.h``, ``include/b200_layernorm.h``
and ``include/b200_softmax.h``
and links the CUDA runtime statically, so the same file serves the ctypes
binding here and any other FFI host.
"""

from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
PRODUCT_DIR = PACKAGE_DIR.parent
REPO_ROOT = PRODUCT_DIR.parent
CSRC = PRODUCT_DIR / "csrc"
INCLUDE = REPO_ROOT / "include"
LIB_NAME = "libb200_attention.so"
LIB_PATH = PACKAGE_DIR / LIB_NAME
# Same source with every TMA coordinate, shared-memory tile address and
# tensor-memory column range checked on the device (for tests; a failed check
# sets B200_ATTN_DEVERR_BOUNDS in the error word instead of faulting).
CHECKED_LIB_PATH = PACKAGE_DIR / "libb200_attention_checked.so"

SOURCES = ("attn_fwd_sm100.cu", "linear_sm100.cu", "layernorm.cu", "softmax.cu")
HEADERS = ("sm100_ptx.cuh", "error_word.cuh", "byte_range.h")

NVCC_FLAGS = (
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler", "-fPIC",
    "-Xcompiler", "-fvisibility=hidden",
    "-shared",
)


def _nvcc() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    candidate = Path(cuda_home) / "bin" / "nvcc"
    if candidate.exists():
        return str(candidate)
    found = shutil.which("nvcc")
    if not found:
        raise RuntimeError("nvcc not found; set CUDA_HOME")
    return found


def _inputs() -> list[Path]:
    files = [CSRC / s for s in SOURCES] + [CSRC / h for h in HEADERS]
    files += [INCLUDE / h for h in ("b200_attn.h", "b200_linear.h", "b200_layernorm.h",
                                    "b200_softmax.h")]
    return files


def is_stale(path: Path = LIB_PATH) -> bool:
    if not path.exists():
        return True
    built = path.stat().st_mtime
    return any(f.stat().st_mtime > built for f in _inputs())


def build_native(force: bool = False, verbose: bool = False, checked: bool = False) -> Path:
    """Compile ``libb200_attention.so`` (or, with ``checked``, the bounds-checked
    ``libb200_attention_checked.so``) next to this file; skipped when fresh."""
    out = CHECKED_LIB_PATH if checked else LIB_PATH
    if not force and not is_stale(out):
        return out
    tmp = out.with_suffix(".so.tmp")
    defines = ["-DB200_ATTN_CHECKED=1"] if checked else []
    cmd = [_nvcc(), *NVCC_FLAGS, *defines, f"-I{INCLUDE}", f"-I{CSRC}",
           *[str(CSRC / s) for s in SOURCES], "-o", str(tmp)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd))
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed ({proc.returncode}):\n{proc.stderr[-8000:]}")
    if verbose and proc.stderr:
        print(proc.stderr)
    os.replace(tmp, out)
    return out


# The attention operator as a torch custom op (torch.ops.b200.fused_attention)
# over the same C ABI: a C++ translation unit against torch's headers, linked
# to libb200_attention.so found next to it ($ORIGIN).
TORCH_OP_SOURCE = CSRC / "torch_op.cpp"
TORCH_OP_PATH = PACKAGE_DIR / "libb200_attention_torch.so"


def _torch_op_stale() -> bool:
    if not TORCH_OP_PATH.exists():
        return True
    built = TORCH_OP_PATH.stat().st_mtime
    deps = (TORCH_OP_SOURCE, INCLUDE / "b200_attn.h", LIB_PATH)
    return any(f.stat().st_mtime > built for f in deps if f.exists())


def build_torch_op(force: bool = False, verbose: bool = False) -> Path:
    """Compile ``libb200_attention_torch.so`` (needs the C-ABI library built
    first); skipped when fresh."""
    if not force and not _torch_op_stale():
        return TORCH_OP_PATH
    import torch
    from torch.utils import cpp_extension

    if not LIB_PATH.exists():
        raise RuntimeError(f"{LIB_PATH.name} must be built before the torch op")
    includes = cpp_extension.include_paths(device_type="cuda") + [str(INCLUDE)]
    libdirs = cpp_extension.library_paths(device_type="cuda")
    torch_lib = str(Path(torch.__file__).resolve().parent / "lib")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    tmp = TORCH_OP_PATH.with_suffix(".so.tmp")
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-fvisibility=hidden",
           f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           *[f"-I{d}" for d in includes], str(TORCH_OP_SOURCE),
           *[f"-L{d}" for d in libdirs], f"-L{PACKAGE_DIR}",
           "-l:libb200_attention.so", "-lc10", "-lc10_cuda", "-ltorch_cpu", "-ltorch",
           "-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{torch_lib}", "-o", str(tmp)]
    if verbose:
        print(" ".join(cmd))
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"g++ failed ({proc.returncode}):\n{proc.stderr[-8000:]}")
    os.replace(tmp, TORCH_OP_PATH)
    return TORCH_OP_PATH


if __name__ == "__main__":
    import sys

    print(build_native(force="--force" in sys.argv, verbose="-v" in sys.argv))
    print(build_native(force="--force" in sys.argv, checked=True))
    print(build_torch_op(force="--force" in sys.argv, verbose="-v" in sys.argv))
