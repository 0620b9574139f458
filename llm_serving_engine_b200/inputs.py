"""Seeded synthetic inputs with the distributions the benchmark configs name.

Drawn on the CPU with `torch.Generator().manual_seed(seed)` in the order x, W, s, so the CPU
baseline, the oracle and the GPU see identical bits:

* x ~ N(0, 1), rounded to bf16, [M, K];
* W uniform on the integers [-127, 127], int8 [N, K] (the nn.Linear [out, in] layout);
* s uniform on [1e-4, 5e-4], fp32 [N] (per output channel); no bias.
"""

from __future__ import annotations

import torch

# Llama-3-8B projection shapes (K, N): fused QKV, O, fused gate_up, down.
LLAMA3_8B_SHAPES = {
    "qkv": (4096, 6144),
    "o": (4096, 4096),
    "gate_up": (4096, 28672),
    "down": (14336, 4096),
}
# Llama-3-70B projection shapes (K, N).
LLAMA3_70B_SHAPES = {
    "qkv": (8192, 10240),
    "o": (8192, 8192),
    "gate_up": (8192, 57344),
    "down": (28672, 8192),
}
DECODE_M = (1, 4, 16, 64)
PREFILL_M = (512, 2048, 8192)


def make_inputs(M: int, K: int, N: int, seed: int = 0):
    """(x bf16 [M,K], W int8 [N,K], s fp32 [N]) on the CPU."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    w = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int8)
    s = torch.empty(N).uniform_(1e-4, 5e-4, generator=g)
    return x, w, s


def linear_bytes(M: int, K: int, N: int) -> int:
    """Algorithmic HBM bytes of one int8 linear: int8 W + fp32 scales + bf16 x + bf16 y."""
    return N * K + 4 * N + 2 * M * K + 2 * M * N


def linear_flops(M: int, K: int, N: int) -> int:
    return 2 * M * N * K
