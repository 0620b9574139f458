"""The C-ABI library builds, loads without a GPU, exports every declared symbol, and rejects
bad arguments on the host before any launch (CPU only)."""

from __future__ import annotations

import ctypes
import os
import re

import pytest

from llm_serving_engine_b200 import _lib, build

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "lse_int8.h")


def declared_functions() -> list[str]:
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(lse_[a-z0-9_]+)\s*\(", text)))


def test_library_builds_and_loads():
    path = build.build()
    assert os.path.exists(path)
    lib = _lib.load()
    assert lib.lse_abi_version() == _lib.ABI_VERSION


def test_every_declared_symbol_is_exported_and_bound():
    lib = _lib.load()
    names = declared_functions()
    assert "lse_int8_linear" in names and "lse_int8_quantize" in names
    for name in names:
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"


def test_header_constants_match_binding():
    text = open(HEADER).read()
    assert int(re.search(r"#define LSE_WS_COUNTER_BYTES (\d+)", text).group(1)) == _lib.WS_COUNTER_BYTES
    assert int(re.search(r"#define LSE_ABI_VERSION (\d+)", text).group(1)) == _lib.ABI_VERSION
    for name, val in [("LSE_ERR_ALIGNMENT", _lib.LSE_ERR_ALIGNMENT), ("LSE_ERR_WORKSPACE", _lib.LSE_ERR_WORKSPACE),
                      ("LSE_ERR_DEVICE_TIMEOUT", _lib.LSE_ERR_DEVICE_TIMEOUT)]:
        assert re.search(rf"{name} = {val}\b", text), name


def test_status_strings():
    for st in range(7):
        assert _lib.status_string(st)
    assert _lib.status_string(99) == "unknown status"


def _call(M=4, K=64, ldx=64, N=32, ldy=32, x=16, w=16, s=16, y=16, ws=16, wsb=1 << 26, algo=0):
    lib = _lib.load()
    return lib.lse_int8_linear_ex(x, M, K, ldx, w, s, N, y, ldy, ws, wsb, algo, None)


def test_host_validation_rejects_before_launch():
    # no device is touched for these: validation precedes every CUDA call
    assert _call(M=-1) == _lib.LSE_ERR_INVALID_ARG
    assert _call(M=0) == _lib.LSE_OK and _call(N=0) == _lib.LSE_OK
    assert _call(x=0) == _lib.LSE_ERR_INVALID_ARG
    assert _call(ldx=32) == _lib.LSE_ERR_INVALID_ARG
    assert _call(ldy=16) == _lib.LSE_ERR_INVALID_ARG
    assert _call(K=24, ldx=24) == _lib.LSE_ERR_ALIGNMENT
    assert _call(ldx=68) == _lib.LSE_ERR_ALIGNMENT
    assert _call(x=24) == _lib.LSE_ERR_ALIGNMENT
    assert _call(w=8) == _lib.LSE_ERR_ALIGNMENT
    assert _call(algo=7) == _lib.LSE_ERR_INVALID_ARG
    assert _call(algo=_lib.ALGO_SKINNY) == _lib.LSE_ERR_UNSUPPORTED  # skinny needs packed W
    lib = _lib.load()
    assert lib.lse_int8_quantize(None, 0, 4, 4, 4, None, None, None) == _lib.LSE_ERR_INVALID_ARG
    assert lib.lse_int8_quantize(16, 0, 4, 8, 4, 16, 16, None) == _lib.LSE_ERR_INVALID_ARG


def test_workspace_size_covers_counter_region():
    lib = _lib.load()
    for M in (1, 16, 17, 64, 65, 8192):
        assert lib.lse_int8_linear_workspace(M, 4096, 4096) > _lib.WS_COUNTER_BYTES
    assert lib.lse_int8_linear_workspace(0, 1, 1) == _lib.WS_COUNTER_BYTES


def test_no_cpu_fallback():
    import torch

    from llm_serving_engine_b200 import ops

    x = torch.zeros(2, 16, dtype=torch.bfloat16)
    w = torch.zeros(4, 16, dtype=torch.int8)
    s = torch.ones(4)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.int8_linear(x, w, s)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.quantize_per_channel(torch.zeros(4, 16))


def test_library_has_no_libcuda_link_dependency():
    """Loads on hosts without a driver: libcuda is reached only through the runtime's
    driver-entry-point query."""
    import subprocess

    deps = subprocess.run(["ldd", build.LIB_PATH], capture_output=True, text=True).stdout
    assert "libcuda.so" not in deps and "libcudart" not in deps, deps
    ctypes.CDLL(build.LIB_PATH)
