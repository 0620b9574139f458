"""ctypes binding of liblse_int8.so, the C ABI declared in include/lse_int8.h.

The library is the only compute path: importing works anywhere (so CPU-only tools can inspect
it), but every call that would launch a kernel raises if the library is missing or CUDA is
unavailable.  There is no CPU fallback.
"""

from __future__ import annotations

import ctypes
import os
import threading

from . import build as _build

LIB_PATH = _build.LIB_PATH

# lse_status codes (include/lse_int8.h)
LSE_OK = 0
LSE_ERR_INVALID_ARG = 1
LSE_ERR_ALIGNMENT = 2
LSE_ERR_UNSUPPORTED = 3
LSE_ERR_WORKSPACE = 4
LSE_ERR_CUDA = 5
LSE_ERR_DEVICE_TIMEOUT = 6

# lse_algo
ALGO_AUTO = 0
ALGO_GEMV = 1
ALGO_TCGEN05 = 2
ALGO_SKINNY = 3

# lse_dtype
DT_BF16 = 0
DT_F16 = 1
DT_F32 = 2

WS_COUNTER_BYTES = 65536
NOALLOC_SCRATCH_BYTES = 16777216  # fixed scratch of lse_int8_linear_packed_noalloc, per device
NOALLOC_MAX_M = 64
GATE_UP_SILU_MAX_M = 16  # lse_int8_gate_up_silu_packed's token range (the decode kernel's)
ABI_VERSION = 1

# Every symbol include/lse_int8.h declares, with its ctypes signature.
_P, _I64, _I32, _SZ = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_size_t
SIGNATURES = {
    "lse_init": ([_I32], _I32),
    "lse_int8_linear": ([_P, _I64, _I64, _I64, _P, _P, _I64, _P, _I64, _P, _SZ, _P], _I32),
    "lse_int8_linear_ex": ([_P, _I64, _I64, _I64, _P, _P, _I64, _P, _I64, _P, _SZ, _I32, _P], _I32),
    "lse_int8_linear_workspace": ([_I64, _I64, _I64], _SZ),
    "lse_int8_linear_workspace_for": ([_I64, _I64, _I64, _I32, _I32], _SZ),
    "lse_int8_linear_packed": ([_P, _I64, _I64, _I64, _P, _P, _I64, _P, _I64, _P, _SZ, _I32, _P], _I32),
    "lse_int8_linear_packed_residual": ([_P, _I64, _I64, _I64, _P, _P, _I64, _P, _I64, _P, _I64, _P, _SZ, _I32, _P],
                                        _I32),
    "lse_int8_linear_packed_noalloc": ([_P, _I64, _I64, _I64, _P, _P, _I64, _P, _I64, _P], _I32),
    "lse_int8_gate_up_silu_packed": ([_P, _I64, _I64, _I64, _P, _P, _I64, _P, _I64, _P], _I32),
    "lse_int8_gate_up_silu_packed_ws": ([_P, _I64, _I64, _I64, _P, _P, _I64, _P, _I64, _P, _SZ, _P], _I32),
    "lse_int8_linear_packed_dt": ([_P, _I32, _I64, _I64, _I64, _P, _P, _I64, _P, _I64, _P, _I64, _P, _SZ, _I32, _P],
                                  _I32),
    "lse_int8_gate_up_silu_packed_dt": ([_P, _I32, _I64, _I64, _I64, _P, _P, _I64, _P, _I64, _P, _SZ, _P], _I32),
    "lse_rms_norm": ([_P, _I64, _I64, _I64, _P, ctypes.c_float, _P, _I64, _P], _I32),
    "lse_int8_rms_norm_proj_workspace": ([_I64, _I64], _SZ),
    "lse_int8_rms_norm_linear_packed": ([_P, _I64, _I64, _I64, _P, ctypes.c_float, _P, _P, _I64, _P, _I64, _P, _SZ, _P],
                                        _I32),
    "lse_int8_rms_norm_gate_up_silu_packed": ([_P, _I64, _I64, _I64, _P, ctypes.c_float, _P, _P, _I64, _P, _I64, _P,
                                               _SZ, _P], _I32),
    "lse_rope_kv_write": ([_P, _I64, _I64, _I64, _I64, _I64, _P, _P, _I64, _I32, _P, _P, _P, _P, _I64, _P], _I32),
    "lse_rope_kv_write_dt": ([_P, _I32, _I64, _I64, _I64, _I64, _I64, _P, _P, _I64, _I32, _P, _P, _P, _P, _I64, _P],
                             _I32),
    "lse_rms_norm_dt": ([_P, _I32, _I64, _I64, _I64, _P, ctypes.c_float, _P, _I64, _P], _I32),
    "lse_paged_decode_attention_workspace": ([_I64, _I64, _I64, _I64, _I64, _I64], _SZ),
    "lse_paged_decode_attention": ([_P, _I64, _I64, _I64, _I64, _I64, _P, _P, _I64, _I64, _I64, _P, _I64, _P, _I64,
                                    ctypes.c_float, _P, _I64, _I64, _P, _SZ, _P], _I32),
    "lse_paged_decode_attention_dt": ([_P, _I32, _I64, _I64, _I64, _I64, _I64, _P, _P, _I64, _I64, _I64, _P, _I64, _P, _I64,
                                    ctypes.c_float, _P, _I64, _I64, _P, _SZ, _P], _I32),
    "lse_int8_packed_weight_bytes": ([_I64, _I64], _SZ),
    "lse_int8_pack_weight": ([_P, _I64, _I64, _I64, _P, _P], _I32),
    "lse_int8_unpack_weight": ([_P, _I64, _I64, _P, _P], _I32),
    "lse_int8_quantize": ([_P, _I32, _I64, _I64, _I64, _P, _P, _P], _I32),
    "lse_status_string": ([_I32], ctypes.c_char_p),
    "lse_last_cuda_error": ([], ctypes.c_char_p),
    "lse_device_status": ([_I32, _I32], _I32),
    "lse_set_wait_limit": ([_I32, ctypes.c_longlong], _I32),
    "lse_paged_attention": ([_P, _I32, _I64, _I64, _I64, _I64, _P, _P, _I64, _I64, _I64, _P, _I64, _P, _P, _P, _P,
                             _I64, _I64, ctypes.c_float, _P, _I64, _I64, _P], _I32),
    "lse_abi_version": ([], _I32),
}

_lib: ctypes.CDLL | None = None
_lock = threading.Lock()


class LseError(RuntimeError):
    """A nonzero lse_status from the library."""

    def __init__(self, status: int, what: str):
        self.status = status
        msg = f"{what}: {status_string(status)} (status {status})"
        detail = last_cuda_error() if status == LSE_ERR_CUDA else ""
        super().__init__(msg + (f": {detail}" if detail else ""))


def load(build_if_missing: bool = True) -> ctypes.CDLL:
    """Load liblse_int8.so (building it in-tree with nvcc if absent)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                if not build_if_missing:
                    raise RuntimeError(f"{LIB_PATH} is missing; run python -m llm_serving_engine_b200.build")
                _build.build()
            lib = ctypes.CDLL(LIB_PATH)
            for name, (args, res) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.argtypes = args
                fn.restype = res
            if lib.lse_abi_version() != ABI_VERSION:
                raise RuntimeError(f"{LIB_PATH}: ABI version {lib.lse_abi_version()} != {ABI_VERSION}")
            _lib = lib
    return _lib


def status_string(status: int) -> str:
    return load().lse_status_string(int(status)).decode()


def last_cuda_error() -> str:
    return load().lse_last_cuda_error().decode()


def check(status: int, what: str) -> None:
    if status != LSE_OK:
        raise LseError(status, what)
