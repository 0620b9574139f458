"""CPU oracle for paged attention (test infrastructure only).

This module is the CHECKER, never the product: only `tests/`, `__graft_entry__.smoke()`
and `bench.py`'s CPU legs may import it.  The shipped path is the sm_100a kernels in
`llm_serving_engine_b200/csrc/decode_attn.cuh` and `paged_attn.cuh`, which fail loudly when
the library is missing instead of falling back to anything here.

What it restates
----------------
The reference's batched attention, `paged_attention_2` / `paged_attention_forward`
(`src/llm_serving_engine/kernels/flash_attention.py:202-332`), for the decode case: one
query token per batch entry (`q_len = 1`) at position `query_offset = context_len - 1`.
K/V live in a shared per-layer pool `(num_blocks, block_size, H_KV, D)`; position `p` of
entry `e` is pool block `block_table[e, p // block_size]`, slot `p % block_size`
(`flash_attention.py:263-271`); only positions `< context_len[e]` are read and the causal
mask lets the query see every one of them (`:276`).  Query head `h` reads KV head
`h // (H // H_KV)` (grouped-query attention, `:240`).  Scores are scaled by
`1 / sqrt(D)` (`:328`) and normalised with a softmax.  Here everything is float64 and the
softmax is the direct formula, not the kernel's online one.
"""

from __future__ import annotations

import numpy as np

__all__ = ["ref_paged_decode_attention", "ref_paged_attention", "gather_kv"]


def gather_kv(pool: np.ndarray, block_table: np.ndarray, e: int, ctx: int) -> np.ndarray:
    """Positions 0..ctx-1 of entry e from a (num_blocks, block_size, H_KV, D) pool:
    (ctx, H_KV, D)."""
    bs = pool.shape[1]
    pos = np.arange(ctx)
    return pool[block_table[e, pos // bs], pos % bs]


def ref_paged_decode_attention(q: np.ndarray, k_pool: np.ndarray, v_pool: np.ndarray,
                               block_table: np.ndarray, context_len: np.ndarray,
                               scale: float | None = None) -> np.ndarray:
    """q (E, H, D) -> o (E, H, D), float64.  An entry with context_len 0 gets zeros."""
    q = np.asarray(q, dtype=np.float64)
    E, H, D = q.shape
    H_kv = k_pool.shape[2]
    G = H // H_kv
    scale = 1.0 / np.sqrt(D) if scale is None else scale
    out = np.zeros((E, H, D), dtype=np.float64)
    for e in range(E):
        ctx = int(context_len[e])
        if ctx == 0:
            continue
        k = gather_kv(k_pool, block_table, e, ctx).astype(np.float64)
        v = gather_kv(v_pool, block_table, e, ctx).astype(np.float64)
        for h in range(H):
            s = k[:, h // G, :] @ q[e, h] * scale
            w = np.exp(s - s.max())
            out[e, h] = (w / w.sum()) @ v[:, h // G, :]
    return out


def ref_paged_attention(q: np.ndarray, k_pool: np.ndarray, v_pool: np.ndarray, block_table: np.ndarray,
                        context_len: np.ndarray, query_offset: np.ndarray, q_start: np.ndarray, q_len: np.ndarray,
                        scale: float | None = None) -> np.ndarray:
    """The general case of `paged_attention_2` (`flash_attention.py:202-284`): q (H, T, D) holds
    every batch entry's query tokens, entry e's rows q_start[e] .. q_start[e] + q_len[e] - 1;
    row i of entry e sits at position query_offset[e] + i and attends to the positions
    p < context_len[e] with p <= query_offset[e] + i (`:276`).  Returns o (H, T, D), float64;
    rows no entry covers stay zero, and so does a row with no position to attend to."""
    q = np.asarray(q, dtype=np.float64)
    H, T, D = q.shape
    H_kv = k_pool.shape[2]
    G = H // H_kv
    scale = 1.0 / np.sqrt(D) if scale is None else scale
    out = np.zeros((H, T, D), dtype=np.float64)
    for e in range(len(q_len)):
        ctx, off, qs, ql = (int(context_len[e]), int(query_offset[e]), int(q_start[e]), int(q_len[e]))
        if ctx == 0 or ql == 0:
            continue
        k = gather_kv(k_pool, block_table, e, ctx).astype(np.float64)
        v = gather_kv(v_pool, block_table, e, ctx).astype(np.float64)
        for i in range(ql):
            n = min(ctx, off + i + 1)
            if n <= 0:
                continue
            for h in range(H):
                s_ = k[:n, h // G, :] @ q[h, qs + i] * scale
                w = np.exp(s_ - s_.max())
                out[h, qs + i] = (w / w.sum()) @ v[:n, h // G, :]
    return out
