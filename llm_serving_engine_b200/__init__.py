"""B200-native (sm_100a) int8 weight-only linear for vladimirfilip/llm-serving-engine.

The compute path is liblse_int8.so (hand-written CUDA for sm_100a, C ABI in
include/lse_int8.h); this package is its host side: the ctypes binding (`_lib`), the
torch-facing ops (`ops`), the drop-in modules (`int8_linear`), the engine hook (`engine`),
the column-split multi-GPU layer (`parallel`) and the seeded inputs (`inputs`).
"""

from .ops import ALGO_AUTO, ALGO_GEMV, ALGO_TCGEN05, device_status, int8_linear, quantize_per_channel  # noqa: F401

__version__ = "0.1.0"
