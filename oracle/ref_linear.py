"""CPU oracle for the int8 weight-only linear (test infrastructure only).

This module is the CHECKER, never the product: only `tests/`, `__graft_entry__.smoke()`
and `bench.py`'s CPU-baseline / reference arm may import it.  The shipped path is the
sm_100a CUDA library under `llm_serving_engine_b200/csrc/`, which fails loudly when it is
missing instead of falling back to anything here.

What it restates
----------------
The reference engine (vladimirfilip/llm-serving-engine) has no int8 linear of its own:
`src/llm_serving_engine/model/model_runner.py:45-46` raises
`NotImplementedError("int8 weight-only quantization")` for `ModelConfig.quantize == "int8"`
(`src/llm_serving_engine/config.py:32,46`).  Every projection it runs is a
`torch.nn.Linear` called at `model_runner.py:322-324` (q/k/v), `:369` and `:418` (o) and
`:223` (the MLP, `down(silu(gate(x)) * up(x))`), with the `nn.Linear` convention
`y = x @ W.T`, weight `[out_features, in_features]`, no bias (Llama).

The int8 layer replaces that weight by `W[n, k] ~= q[n, k] * s[n]` with `q` int8 and `s`
fp32 per output channel, so the oracle is the dequant-matmul

    y[m, n] = sum_k x[m, k] * (q[n, k] * s[n])           (float64 here)

and parity of the oracle with the reference is pinned by fixtures captured from the
reference's own `nn.Linear` CPU path (`model_runner.py:185-200`, `_forward_hf`) run on the
dequantized weights (`tests/golden/make_golden.py`).

Quantization (`ref_quantize`) has no reference counterpart (the reference raises before it
would quantize); it restates the symmetric per-output-channel rule
`s[n] = max_k |W[n, k]| / 127`, `q = clamp(rint(W / s), -127, 127)` in float32 arithmetic,
step for step as the CUDA kernel does it, so the two agree bit for bit.
"""

from __future__ import annotations

import numpy as np

__all__ = [
    "bf16_bits_to_f32",
    "f32_to_bf16_bits",
    "ref_int8_linear",
    "ref_quantize",
    "ref_pack_weight",
    "ref_fused_split",
    "ref_mlp",
    "parity_errors",
    "NORMWISE_TOL",
    "ELEMWISE_RTOL",
    "ELEMWISE_ATOL_FRAC",
]

# Pass criterion for a bf16-output kernel against this oracle (north_star: max relative error
# 1e-2 against an fp32 dequant-matmul oracle).  Normwise: max|y-ref| / max|ref|.
# Elementwise: |y-ref| <= ELEMWISE_RTOL*|ref| + ELEMWISE_ATOL_FRAC*max|ref|.
NORMWISE_TOL = 1e-2
ELEMWISE_RTOL = 1e-2
ELEMWISE_ATOL_FRAC = 1e-3


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    """uint16 bfloat16 bit patterns -> float32 (exact)."""
    bits = np.asarray(bits, dtype=np.uint16)
    return (bits.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bfloat16 bit patterns, round to nearest even (NaN kept quiet)."""
    u = np.asarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    rounding = ((u >> 16) & 1) + 0x7FFF
    out = ((u + rounding) >> 16).astype(np.uint16)
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    out[nan] = 0x7FC0
    return out


def ref_int8_linear(x: np.ndarray, q: np.ndarray, s: np.ndarray) -> np.ndarray:
    """y = x @ (q * s[:, None]).T in float64.

    x: [..., K] float (bf16 values already widened, or fp32); q: int8 [N, K]; s: [N].
    Returns float64 [..., N].  Follows the nn.Linear convention of
    `model_runner.py:322-324` (weight [out, in], y = x W^T, no bias).
    """
    x64 = np.asarray(x, dtype=np.float64)
    w64 = np.asarray(q, dtype=np.int8).astype(np.float64) * np.asarray(s, np.float64)[:, None]
    return x64 @ w64.T


def ref_quantize(w: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Symmetric per-output-channel int8 quantization of W [N, K] (float32 arithmetic).

    amax[n] = max_k |W[n,k]|; s[n] = amax[n] / 127 (fp32 division, round to nearest),
    or 1.0 for an all-zero row; q[n,k] = clamp(rint(W[n,k] / s[n]), -127, 127) with the
    division in fp32 and rint = round half to even.
    """
    w32 = np.asarray(w, dtype=np.float32)
    amax = np.max(np.abs(w32), axis=1) if w32.shape[1] else np.zeros(w32.shape[0], np.float32)
    s = (amax / np.float32(127.0)).astype(np.float32)
    s = np.where(s > 0, s, np.float32(1.0)).astype(np.float32)
    with np.errstate(invalid="ignore", over="ignore"):
        r = np.rint((w32 / s[:, None]).astype(np.float32))
    q = np.clip(r, -127, 127).astype(np.int8)
    return q, s


def ref_fused_split(y: np.ndarray, sizes: list[int]) -> list[np.ndarray]:
    """Column split of a fused projection's output: QKV -> (q, k, v) with sizes
    (n_heads*hd, n_kv*hd, n_kv*hd) as `model_runner.py:320-324` shapes them, or
    gate_up -> (gate, up)."""
    out, start = [], 0
    for n in sizes:
        out.append(y[..., start:start + n])
        start += n
    assert start == y.shape[-1]
    return out


def ref_mlp(x: np.ndarray, q_gate, s_gate, q_up, s_up, q_down, s_down) -> np.ndarray:
    """Llama MLP `down(silu(gate(x)) * up(x))` (transformers' LlamaMLP.forward, reached at
    `model_runner.py:223`) with each projection the int8 dequant-matmul, in float64."""
    g = ref_int8_linear(x, q_gate, s_gate)
    u = ref_int8_linear(x, q_up, s_up)
    h = (g / (1.0 + np.exp(-g))) * u
    return ref_int8_linear(h, q_down, s_down)


def ref_pack_weight(q: np.ndarray) -> np.ndarray:
    """The build's packed weight layout, restated with numpy (checker for the pack kernel).
    W is zero padded to multiples of 128 in both dimensions and cut into row blocks of 16
    rows; row block b is a run of 16*Kp bytes of 2 KB blocks, one per 128 columns, each holding
    the block's two 8-row groups (h) one after the other as two 512-byte atoms of 64 columns
    (a), an atom holding its 8 rows' 64 columns 64 bytes per row with the 16-byte chunk c of row
    r stored at chunk position c ^ ((r >> 1) & 3) (plain two's-complement bytes):
    W[16b + 8h + r][128t + 64a + 16c + e] at
    b*16*Kp + t*2048 + h*1024 + a*512 + r*64 + (c ^ ((r >> 1) & 3))*16 + e."""
    N, K = q.shape
    Np, Kp = -(-N // 128) * 128, -(-K // 128) * 128
    pad = np.zeros((Np, Kp), dtype=np.int8)
    pad[:N, :K] = q
    # axes: b, h, r, t, a, c, e  ->  b, t, h, a, r, c', e  (stored chunk position c' = c ^ ((r >> 1) & 3))
    v = pad.reshape(Np // 16, 2, 8, Kp // 128, 2, 4, 16).transpose(0, 3, 1, 4, 2, 5, 6)
    out = np.empty_like(v)
    for r in range(8):
        out[:, :, :, :, r, np.arange(4) ^ ((r >> 1) & 3), :] = v[:, :, :, :, r, :, :]
    return out.reshape(-1)


def parity_errors(y: np.ndarray, ref: np.ndarray) -> tuple[float, bool, float]:
    """(normwise max|y-ref|/max|ref|, elementwise criterion holds, worst elementwise ratio).

    The elementwise ratio is max |y-ref| / (RTOL*|ref| + ATOL_FRAC*max|ref|); the criterion
    holds when it is <= 1.
    """
    y64 = np.asarray(y, dtype=np.float64)
    r64 = np.asarray(ref, dtype=np.float64)
    if r64.size == 0:
        return 0.0, True, 0.0
    diff = np.abs(y64 - r64)
    scale = float(np.max(np.abs(r64)))
    if scale == 0.0:
        worst = float(np.max(diff))
        return worst, worst == 0.0, worst
    normwise = float(np.max(diff)) / scale
    bound = ELEMWISE_RTOL * np.abs(r64) + ELEMWISE_ATOL_FRAC * scale
    ratio = float(np.max(diff / bound))
    return normwise, ratio <= 1.0, ratio
