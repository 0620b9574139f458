"""In-tree build of the sm_100a CUDA library (liblse_int8.so) with nvcc.

`python -m llm_serving_engine_b200.build` (or `build()`) compiles
`csrc/lse_int8.cu` into `llm_serving_engine_b200/_lib/liblse_int8.so`, a plain C-ABI shared
library (static CUDA runtime, no torch, no link-time libcuda).  The build is skipped when
the library is newer than every source and header.
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


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
