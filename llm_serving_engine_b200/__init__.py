"""B200-native (sm_100a) int8 weight-only linear for vladimirfilip/llm-serving-engine.

The compute path is liblse_int8.so (hand-written CUDA for sm_100a, C ABI in
include/lse_int8.h); this package is its host side: the ctypes binding (`_lib`), the
torch-facing ops (`ops`), the drop-in modules and the model hook (`int8_linear`), the
on-disk int8 checkpoint (`checkpoint`), the output-column split over ranks (`parallel`)
and the seeded inputs (`inputs`).
"""

from .checkpoint import load_int8_checkpoint_, save_int8_checkpoint  # noqa: F401
from .int8_linear import FusedInt8QKV, Int8Linear, Int8LlamaMLP, int8_weight_bytes, quantize_llama_  # noqa: F401
from .ops import (ALGO_AUTO, ALGO_GEMV, ALGO_SKINNY, ALGO_TCGEN05, device_status, int8_linear,  # noqa: F401
                  int8_linear_packed, pack_weight, quantize_per_channel)

__version__ = "0.1.0"
