"""CPU oracle for the int8 linear: test infrastructure, never the shipped path.

Importable only from tests/, __graft_entry__.smoke() and bench.py's CPU legs.
"""

from .ref_linear import (  # noqa: F401
    ELEMWISE_ATOL_FRAC,
    ELEMWISE_RTOL,
    NORMWISE_TOL,
    bf16_bits_to_f32,
    f32_to_bf16_bits,
    parity_errors,
    ref_fused_split,
    ref_int8_linear,
    ref_mlp,
    ref_quantize,
)
