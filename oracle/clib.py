"""ctypes binding of the plain-C oracle (oracle/_build/liboracle.so). Test infrastructure."""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "liboracle.so")
_lib = None


def build() -> str:
    """Compile the C oracle with its Makefile (no-op when up to date)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        _lib = ctypes.CDLL(_LIB_PATH)
        p = ctypes.c_void_p
        i64 = ctypes.c_int64
        _lib.oracle_int8_linear_f64.argtypes = [p, i64, i64, i64, p, p, i64, p]
        _lib.oracle_int8_linear_f64.restype = None
        _lib.oracle_quantize_f32.argtypes = [p, i64, i64, p, p]
        _lib.oracle_quantize_f32.restype = None
    return _lib


def c_int8_linear(x: np.ndarray, q: np.ndarray, s: np.ndarray) -> np.ndarray:
    """float64 [M, N] from the C triple loop; x float32 [M, K]."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    q = np.ascontiguousarray(q, dtype=np.int8)
    s = np.ascontiguousarray(s, dtype=np.float32)
    M, K = x.shape
    N = q.shape[0]
    y = np.empty((M, N), dtype=np.float64)
    lib().oracle_int8_linear_f64(x.ctypes.data, M, K, K, q.ctypes.data, s.ctypes.data, N,
                                 y.ctypes.data)
    return y


def c_quantize(w: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    w = np.ascontiguousarray(w, dtype=np.float32)
    N, K = w.shape
    q = np.empty((N, K), dtype=np.int8)
    s = np.empty((N,), dtype=np.float32)
    lib().oracle_quantize_f32(w.ctypes.data, N, K, q.ctypes.data, s.ctypes.data)
    return q, s
