"""Host-side logic of the package that needs no GPU: row orders of the fused gate/up weight,
pool slot offsets, and the decode harness's byte count (CPU only)."""

from __future__ import annotations

import pytest
import torch

from llm_serving_engine_b200 import ops
from llm_serving_engine_b200.llama_decode import LLAMA3_8B, LlamaShape, decode_bytes_per_step


def test_interleave_gate_up_rows_order():
    I = 24
    perm = ops.interleave_gate_up_rows(I)
    expect = []
    for j in range(I // 8):
        expect += list(range(8 * j, 8 * j + 8)) + list(range(I + 8 * j, I + 8 * j + 8))
    assert perm.tolist() == expect
    assert sorted(perm.tolist()) == list(range(2 * I))  # a permutation of [gate; up]
    with pytest.raises(ValueError):
        ops.interleave_gate_up_rows(20)


def test_interleaved_weight_pairs_gate_and_up_rows_in_16_row_blocks():
    """Row 16b + r of the interleaved weight is gate row 8b + r for r < 8 and the matching up
    row for r >= 8: the pairing both fused kernels rely on."""
    I, K = 32, 4
    gate = torch.arange(I * K).view(I, K)
    up = -torch.arange(I * K).view(I, K) - 1
    w = torch.cat([gate, up]).index_select(0, ops.interleave_gate_up_rows(I))
    for b in range(I // 8):
        for r in range(8):
            assert torch.equal(w[16 * b + r], gate[8 * b + r])
            assert torch.equal(w[16 * b + 8 + r], up[8 * b + r])


def test_pool_slot_offsets():
    pool = torch.empty(10, 16, 8, 128)  # [num_blocks, block_size, H_kv, D]
    blk = torch.tensor([3, 0, 9], dtype=torch.int32)
    within = torch.tensor([0, 15, 7], dtype=torch.int32)
    off = ops.pool_slot_offsets(blk, within, pool)
    assert off.dtype == torch.int64
    assert off.tolist() == [(3 * 16 + 0) * 1024, (0 * 16 + 15) * 1024, (9 * 16 + 7) * 1024]
    # the offset addresses element (block, within, 0, 0) of the contiguous pool
    flat = torch.arange(pool.numel()).view(pool.shape)
    assert flat[9, 7, 0, 0].item() == off[2].item()


def test_decode_bytes_per_step_counts_weights_kv_head_and_embedding():
    tiny = LlamaShape(layers=2, hidden=64, heads=4, kv_heads=2, head_dim=16, intermediate=128, vocab=100)
    B, ctx = 3, 10
    n_qkv = (4 + 2 * 2) * 16
    shapes = [(64, n_qkv), (64, 64), (64, 256), (128, 64)]  # (K, N) of qkv, o, gate_up, down
    w8 = sum(k * n + 4 * n for k, n in shapes) * 2
    w16 = sum(k * n * 2 for k, n in shapes) * 2
    kv = 2 * 2 * B * 2 * (ctx + 1) * 16 * 2
    emb = B * 64 * 2
    assert decode_bytes_per_step(tiny, B, ctx, True) == w8 + kv + 100 * 64 * 2 + emb
    assert decode_bytes_per_step(tiny, B, ctx, False) == w16 + kv + 100 * 64 * 2 + emb
    assert decode_bytes_per_step(tiny, B, ctx, True, int8_lm_head=True) == w8 + kv + 100 * 64 + 4 * 100 + emb
    # Llama-3-8B int8 projections: 6.98 GB of weights (plus scales) per step
    full = decode_bytes_per_step(LLAMA3_8B, 1, 0, True) - 2 * LLAMA3_8B.layers * 8 * 128 * 2 \
        - LLAMA3_8B.vocab * LLAMA3_8B.hidden * 2 - LLAMA3_8B.hidden * 2
    assert 6.9e9 < full < 7.1e9
