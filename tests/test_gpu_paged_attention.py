"""Multi-token paged attention (sm_100a kernel, `ops.paged_attention`) against the fp64 oracle
restating the reference's `paged_attention_2`, and both attention kernels against the
reference's own Triton `paged_attention_forward` (`kernels/flash_attention.py:287-332`, from
its install in baseline/_ref) on the same inputs.

Cases: mixed batches (fresh prefills, chunks after a cached prefix, single-token decodes),
GQA group sizes 1-8, head_dim 64 and 128, bf16 and fp16, block sizes 16 and 32, shuffled block
tables, key ranges over many 64-position tiles, q and o as the engine's strided views, rows of
no entry left untouched, determinism, and an out-of-range block id reported on the device
status word without a fault.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from llm_serving_engine_b200 import _lib, ops
from oracle.ref_attention import ref_paged_attention
from tests.gpu_helpers import check_parity

pytestmark = pytest.mark.gpu


def _batch(q_len, query_offset, H, H_kv, D, bs, dtype, seed, gap=1):
    """Entries' rows packed with `gap` unused rows before each (rows of no entry)."""
    g = torch.Generator().manual_seed(seed)
    q_len = np.asarray(q_len)
    query_offset = np.asarray(query_offset)
    ctx = query_offset + q_len
    q_start = np.zeros_like(q_len)
    row = 0
    for e, n in enumerate(q_len):
        row += gap
        q_start[e] = row
        row += n
    T = row + gap
    E = len(q_len)
    nbps = max(1, int(-(-ctx.max() // bs)))
    nb = E * nbps + 3
    bt = torch.randperm(nb, generator=g)[: E * nbps].view(E, nbps).to(torch.int32)
    k_pool = torch.randn(nb, bs, H_kv, D, generator=g).to(dtype)
    v_pool = torch.randn(nb, bs, H_kv, D, generator=g).to(dtype)
    q = (torch.randn(H, T, D, generator=g) * 2).to(dtype)
    i32 = lambda a: torch.as_tensor(np.asarray(a), dtype=torch.int32)
    return dict(q=q, k_pool=k_pool, v_pool=v_pool, block_table=bt, context_len=i32(ctx),
                query_offset=i32(query_offset), q_start=i32(q_start), q_len=i32(q_len), block_size=bs,
                max_q_len=int(q_len.max()))


def _cuda(b):
    return {k: (v.cuda() if isinstance(v, torch.Tensor) else v) for k, v in b.items()}


def _oracle(b):
    f = lambda t: t.float().numpy()
    return ref_paged_attention(f(b["q"]), f(b["k_pool"]), f(b["v_pool"]), b["block_table"].numpy(),
                               b["context_len"].numpy(), b["query_offset"].numpy(), b["q_start"].numpy(),
                               b["q_len"].numpy())


def _rows(b):
    return np.concatenate([np.arange(s, s + n) for s, n in zip(b["q_start"].numpy(), b["q_len"].numpy())])


CASES = [
    # q_len, query_offset, H, H_kv, D, bs
    ([37], [0], 32, 8, 128, 16),                                # one fresh prefill chunk
    ([1, 1, 9, 64, 1], [5, 300, 0, 100, 1024], 32, 8, 128, 16),  # mixed decodes and chunks
    ([200, 3], [700, 0], 64, 8, 128, 16),                       # G = 8 (Llama-3-70B), long prefix
    ([17, 33], [12, 96], 16, 8, 128, 32),                       # G = 2, block_size 32
    ([65, 1, 40], [0, 63, 190], 8, 8, 64, 16),                  # G = 1, head_dim 64
    ([129], [1000], 8, 2, 64, 16),                              # G = 4, many key tiles
]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("q_len,query_offset,H,H_kv,D,bs", CASES)
def test_paged_attention_parity(q_len, query_offset, H, H_kv, D, bs, dtype):
    b = _batch(q_len, query_offset, H, H_kv, D, bs, dtype, seed=sum(q_len) + H + D)
    d = _cuda(b)
    sentinel = torch.full_like(d["q"], 7.0)
    o = ops.paged_attention(**d, out=sentinel.clone())
    torch.cuda.synchronize()
    ref = _oracle(b)
    rows = _rows(b)
    H_, T, D_ = o.shape
    check_parity(o[:, rows].reshape(-1, D_), ref[:, rows].reshape(-1, D_), f"paged attention {q_len} G={H // H_kv} D={D}")
    untouched = np.setdiff1d(np.arange(T), rows)
    assert torch.all(o[:, untouched] == 7.0), "a row of no entry was written"
    assert ops.device_status() == _lib.LSE_OK
    o2 = ops.paged_attention(**d, out=sentinel.clone())
    assert torch.equal(o, o2), "not deterministic"


def test_paged_attention_on_the_engines_strided_views():
    """q as the engine hands it over: (1, M, H, D) transposed to (H, M, D) (row stride H * D),
    and an output written into a wider buffer's column slice."""
    b = _batch([5, 1, 12], [3, 40, 0], 32, 8, 128, 16, torch.bfloat16, seed=5, gap=0)
    d = _cuda(b)
    H, T, D = d["q"].shape
    q_view = d["q"].permute(1, 0, 2).contiguous().unsqueeze(0).transpose(1, 2)[0]  # (H, T, D), strides (D, H*D, 1)
    assert q_view.stride() == (D, H * D, 1)
    out_buf = torch.zeros(H, T + 5, D, dtype=torch.bfloat16, device="cuda")
    o = ops.paged_attention(q_view, d["k_pool"], d["v_pool"], d["block_table"], d["context_len"], d["query_offset"],
                            d["q_start"], d["q_len"], d["block_size"], d["max_q_len"], out=out_buf[:, 2:2 + T])
    torch.cuda.synchronize()
    ref = _oracle(b)
    check_parity(o.reshape(-1, D), ref.reshape(-1, D), "strided q / o")
    assert torch.all(out_buf[:, :2] == 0) and torch.all(out_buf[:, 2 + T:] == 0)


def test_paged_attention_bad_block_id_is_reported_not_read():
    b = _batch([4, 1], [20, 7], 8, 2, 64, 16, torch.bfloat16, seed=9)
    b["block_table"][0, 1] = 10_000_000  # positions 16..31 of entry 0
    d = _cuda(b)
    ops.paged_attention(**d)
    assert ops.device_status() == _lib.LSE_ERR_INVALID_ARG
    assert ops.device_status() == _lib.LSE_OK


# ---- against the reference's own Triton kernel ------------------------------------------
def _reference_forward():
    fa = pytest.importorskip("llm_serving_engine.kernels.flash_attention",
                             reason="the reference is installed into baseline/_ref by __graft_entry__.build()")
    return fa.paged_attention_forward


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("q_len,query_offset,H,H_kv,D,bs", CASES[:4])
def test_paged_attention_matches_reference_triton(q_len, query_offset, H, H_kv, D, bs, dtype):
    forward = _reference_forward()
    b = _batch(q_len, query_offset, H, H_kv, D, bs, dtype, seed=3 + sum(q_len), gap=0)
    d = _cuda(b)
    theirs = forward(d["q"], d["k_pool"], d["v_pool"], d["block_table"], d["context_len"], d["query_offset"],
                     d["q_start"], d["q_len"], d["block_size"], d["max_q_len"])
    ours = ops.paged_attention(**d)
    torch.cuda.synchronize()
    rows = _rows(b)
    Dd = ours.shape[-1]
    check_parity(ours[:, rows].reshape(-1, Dd), theirs[:, rows].float().cpu().numpy().reshape(-1, Dd),
                 f"ours vs reference Triton {q_len}")
    # both against the fp64 oracle, ours no further from it than the reference's kernel (+ slack)
    ref = _oracle(b)[:, rows].reshape(-1, Dd)
    err = lambda y: float(np.abs(y[:, rows].float().cpu().numpy().reshape(-1, Dd) - ref).max() / np.abs(ref).max())
    assert err(ours) <= err(theirs) * 1.5 + 1e-3


@pytest.mark.parametrize("E,H,H_kv,D,bs,ctx", [
    (4, 32, 8, 128, 16, [1, 17, 300, 1024]),
    (64, 32, 8, 128, 16, list(range(962, 1026))),
    (3, 8, 8, 64, 8, [5, 129, 64]),
])
def test_decode_attention_matches_reference_triton(E, H, H_kv, D, bs, ctx):
    """The decode kernel (`ops.paged_decode_attention`, one query token per sequence) against
    the reference's Triton kernel at q_len = 1, query_offset = context_len - 1."""
    forward = _reference_forward()
    b = _batch([1] * E, np.asarray(ctx) - 1, H, H_kv, D, bs, torch.bfloat16, seed=E + D, gap=0)
    d = _cuda(b)
    theirs = forward(d["q"], d["k_pool"], d["v_pool"], d["block_table"], d["context_len"], d["query_offset"],
                     d["q_start"], d["q_len"], d["block_size"], 1)
    q_dec = d["q"].transpose(0, 1)  # (E, H, D), strides (D, E*D... ) as a view
    ours = ops.paged_decode_attention(q_dec, d["k_pool"], d["v_pool"], d["block_table"], d["context_len"],
                                      int(max(ctx)))
    torch.cuda.synchronize()
    check_parity(ours.reshape(-1, D), theirs.transpose(0, 1).float().cpu().numpy().reshape(-1, D),
                 f"decode kernel vs reference Triton E={E}")
