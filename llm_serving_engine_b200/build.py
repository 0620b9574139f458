"""In-tree build of the sm_100a CUDA library (liblse_int8.so) with nvcc, and of the torch
operators over it (liblse_torch.so) with the host C++ compiler.

`python -m llm_serving_engine_b200.build` (or `build()`) compiles
`csrc/lse_int8.cu` into `llm_serving_engine_b200/_lib/liblse_int8.so`, a plain C-ABI shared
library (static CUDA runtime, no torch, no link-time libcuda), then `csrc/torch_ops.cpp` into
`_lib/liblse_torch.so` (the `lse::int8_linear` / `lse::gate_up_silu` operators, linked to the
first by a relative run path).  Each build is skipped when its output is newer than every
source and header it reads.
"""

from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
OUT_DIR = os.path.join(PKG_DIR, "_lib")
LIB_PATH = os.path.join(OUT_DIR, "liblse_int8.so")

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build liblse_int8.so")
    return cand


def _sources() -> list[str]:
    files = glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cuh"))
    files.append(os.path.join(REPO_DIR, "include", "lse_int8.h"))
    return files


def up_to_date() -> bool:
    if not os.path.exists(LIB_PATH):
        return False
    t = os.path.getmtime(LIB_PATH)
    return all(os.path.getmtime(f) <= t for f in _sources())


def build(force: bool = False, verbose: bool = False, extra: list[str] | None = None) -> str:
    if not force and up_to_date():
        return LIB_PATH
    os.makedirs(OUT_DIR, exist_ok=True)
    tmp = LIB_PATH + ".tmp"
    cmd = [
        nvcc_path(), *ARCH_FLAGS, "-O3", "-lineinfo", "-std=c++17",
        "-Xcompiler", "-fPIC", "-shared", "-cudart", "static",
        "-Xptxas", "-warn-spills",
        "-I", os.path.join(REPO_DIR, "include"),
        os.path.join(CSRC, "lse_int8.cu"), "-o", tmp,
    ] + (extra or [])
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if verbose and (res.stdout or res.stderr):
        print(res.stdout, res.stderr, file=sys.stderr)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


TORCH_LIB_PATH = os.path.join(OUT_DIR, "liblse_torch.so")


def torch_ops_up_to_date() -> bool:
    if not os.path.exists(TORCH_LIB_PATH):
        return False
    t = os.path.getmtime(TORCH_LIB_PATH)
    deps = [os.path.join(CSRC, "torch_ops.cpp"), os.path.join(REPO_DIR, "include", "lse_int8.h"), LIB_PATH]
    return all(os.path.getmtime(f) <= t for f in deps)


def build_torch_ops(force: bool = False, verbose: bool = False) -> str:
    """liblse_torch.so: the torch.library operators, against this interpreter's torch."""
    if not force and torch_ops_up_to_date():
        return TORCH_LIB_PATH
    import torch
    from torch.utils import cpp_extension as ext

    try:
        incs = ext.include_paths(device_type="cuda")
        libs = ext.library_paths(device_type="cuda")
    except TypeError:  # older signature
        incs = ext.include_paths(cuda=True)
        libs = ext.library_paths(cuda=True)
    torch_lib = os.path.join(os.path.dirname(torch.__file__), "lib")
    abi = 1 if torch.compiled_with_cxx11_abi() else 0
    tmp = TORCH_LIB_PATH + ".tmp"
    cmd = [shutil.which("g++") or "g++", "-O2", "-std=c++17", "-shared", "-fPIC", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           *(f"-I{d}" for d in incs), os.path.join(CSRC, "torch_ops.cpp"), "-o", tmp,
           *(f"-L{d}" for d in libs), f"-L{OUT_DIR}", "-llse_int8", "-lc10", "-lc10_cuda", "-ltorch_cpu", "-ltorch",
           "-ltorch_cuda", "-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{torch_lib}"]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"g++ failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, TORCH_LIB_PATH)
    return TORCH_LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
    print(build_torch_ops(force="--force" in sys.argv, verbose=True))
