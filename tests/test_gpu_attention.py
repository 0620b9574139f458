"""Paged decode attention (sm_100a kernel) against the fp64 oracle restating the reference's
`paged_attention_2` for one query token per sequence: GQA group sizes 1-8, head_dim 64 and
128, ragged context lengths (0, 1, block boundaries, long), shuffled block tables, the
split-K path (few sequences) and the single-pass path (many), determinism, graph replay, and
an out-of-range block id reported on the device status word without a fault."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from llm_serving_engine_b200 import _lib, ops
from oracle.ref_attention import ref_paged_decode_attention
from tests.gpu_helpers import check_parity

pytestmark = pytest.mark.gpu


def _case(E, H, H_kv, D, bs, ctx, seed=0, spare_blocks=3):
    g = torch.Generator().manual_seed(seed)
    ctx = np.asarray(ctx, dtype=np.int64)
    max_ctx = int(ctx.max())
    nbps = max(1, -(-max_ctx // bs))
    nb = E * nbps + spare_blocks
    perm = torch.randperm(nb, generator=g)[: E * nbps].view(E, nbps).to(torch.int32)  # shuffled blocks
    k_pool = (torch.randn(nb, bs, H_kv, D, generator=g)).to(torch.bfloat16)
    v_pool = (torch.randn(nb, bs, H_kv, D, generator=g)).to(torch.bfloat16)
    q = (torch.randn(E, H, D, generator=g) * 2).to(torch.bfloat16)
    return q, k_pool, v_pool, perm, torch.as_tensor(ctx, dtype=torch.int32), max_ctx


def _run(q, k_pool, v_pool, bt, ctx, max_ctx):
    return ops.paged_decode_attention(q.cuda(), k_pool.cuda(), v_pool.cuda(), bt.cuda(), ctx.cuda(), max_ctx)


@pytest.mark.parametrize("E,H,H_kv,D,bs,ctx", [
    (1, 32, 8, 128, 16, [1025]),                       # one sequence: many splits
    (4, 32, 8, 128, 16, [1, 17, 300, 1024]),           # ragged, block boundaries
    (64, 32, 8, 128, 16, list(range(962, 1026))),      # Llama-3-8B decode batch
    (3, 8, 8, 64, 8, [0, 5, 129]),                     # G = 1, head_dim 64, an empty context
    (2, 64, 8, 128, 16, [700, 33]),                    # G = 8 (Llama-3-70B)
    (5, 16, 8, 128, 32, [31, 32, 33, 64, 1000]),       # G = 2, block_size 32
    (6, 8, 2, 64, 16, [4096, 1, 2048, 15, 16, 3000]),  # long contexts, G = 4
])
def test_paged_decode_attention_parity(E, H, H_kv, D, bs, ctx):
    q, k_pool, v_pool, bt, cl, max_ctx = _case(E, H, H_kv, D, bs, ctx, seed=E + H + D)
    o = _run(q, k_pool, v_pool, bt, cl, max_ctx)
    torch.cuda.synchronize()
    ref = ref_paged_decode_attention(q.float().numpy(), k_pool.float().numpy(), v_pool.float().numpy(),
                                     bt.numpy(), cl.numpy())
    check_parity(o.reshape(E * H, D), ref.reshape(E * H, D), f"attention E={E} H={H}/{H_kv} D={D} bs={bs}")
    empty = np.where(cl.numpy() == 0)[0]
    if len(empty):
        assert torch.all(o[torch.as_tensor(empty)] == 0)
    assert ops.device_status() == 0
    o2 = _run(q, k_pool, v_pool, bt, cl, max_ctx)
    torch.cuda.synchronize()
    assert torch.equal(o, o2), "not deterministic"


def test_strided_q_and_out():
    q, k_pool, v_pool, bt, cl, max_ctx = _case(3, 32, 8, 128, 16, [10, 400, 77], seed=5)
    big = torch.zeros(3, 48, 128, dtype=torch.bfloat16, device="cuda")
    big[:, :32] = q.cuda()
    out = torch.full((3, 40, 128), 7.0, dtype=torch.bfloat16, device="cuda")
    ops.paged_decode_attention(big[:, :32], k_pool.cuda(), v_pool.cuda(), bt.cuda(), cl.cuda(), max_ctx,
                               out=out[:, :32])
    ref = _run(q, k_pool, v_pool, bt, cl, max_ctx)
    torch.cuda.synchronize()
    assert torch.equal(out[:, :32], ref)
    assert torch.all(out[:, 32:] == 7.0)


def test_graph_replay_matches_eager():
    q, k_pool, v_pool, bt, cl, max_ctx = _case(8, 32, 8, 128, 16, [1025] * 8, seed=9)
    q, k_pool, v_pool, bt, cl = q.cuda(), k_pool.cuda(), v_pool.cuda(), bt.cuda(), cl.cuda()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        ops.paged_decode_attention(q, k_pool, v_pool, bt, cl, max_ctx)  # workspace for this stream
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=side):
        out = ops.paged_decode_attention(q, k_pool, v_pool, bt, cl, max_ctx)
    for trial in range(3):
        q.copy_(torch.randn_like(q, dtype=torch.float32).to(torch.bfloat16))
        cl.copy_(torch.randint(1, 1026, (8,), dtype=torch.int32, device="cuda"))
        g.replay()
        eager = ops.paged_decode_attention(q, k_pool, v_pool, bt, cl, max_ctx)
        torch.cuda.synchronize()
        assert torch.equal(out, eager), trial


def test_bad_block_id_is_reported_not_read():
    q, k_pool, v_pool, bt, cl, max_ctx = _case(2, 8, 2, 64, 16, [40, 40], seed=3)
    bt[1, 1] = 10_000  # outside the pool
    ops.device_status()  # clear
    _run(q, k_pool, v_pool, bt, cl, max_ctx)
    assert ops.device_status() == _lib.LSE_ERR_INVALID_ARG
    assert ops.device_status() == 0


def test_argument_errors():
    q, k_pool, v_pool, bt, cl, max_ctx = _case(2, 12, 8, 128, 16, [5, 6])  # H % H_kv != 0
    with pytest.raises(_lib.LseError):
        _run(q, k_pool, v_pool, bt, cl, max_ctx)
    q, k_pool, v_pool, bt, cl, max_ctx = _case(2, 8, 8, 96, 16, [5, 6])  # head_dim 96
    with pytest.raises(_lib.LseError):
        _run(q, k_pool, v_pool, bt, cl, max_ctx)
    q, k_pool, v_pool, bt, cl, max_ctx = _case(2, 8, 8, 64, 16, [5, 6])
    with pytest.raises(ValueError):
        ops.paged_decode_attention(q.cuda(), k_pool.cuda(), v_pool.cuda(), bt.cuda().long(), cl.cuda(), max_ctx)


# ---- RoPE + K/V write on the fused QKV output ------------------------------------------
def _rope_ref(x, cos, sin):
    """transformers' rotate-half RoPE in fp32: x [M, heads, D], cos/sin [M, D]."""
    half = x.shape[-1] // 2
    rot = torch.cat([-x[..., half:], x[..., :half]], dim=-1)
    return x * cos[:, None, :] + rot * sin[:, None, :]


@pytest.mark.parametrize("M,H,H_kv,D,cs_dtype,dtype", [
    (1, 32, 8, 128, torch.float32, torch.bfloat16), (7, 32, 8, 128, torch.bfloat16, torch.bfloat16),
    (64, 8, 2, 64, torch.float32, torch.bfloat16), (130, 4, 4, 128, torch.bfloat16, torch.bfloat16),
    (9, 32, 8, 128, torch.float16, torch.float16), (64, 8, 2, 64, torch.float32, torch.float16)])
def test_rope_kv_write_matches_torch(M, H, H_kv, D, cs_dtype, dtype):
    g = torch.Generator().manual_seed(M + H)
    qkv = torch.randn(M, (H + 2 * H_kv) * D, generator=g).to(dtype).cuda()
    pos = torch.randint(0, 4096, (M,), generator=g).float()
    inv = 1.0 / (500000.0 ** (torch.arange(0, D, 2).float() / D))
    ang = pos[:, None] * inv[None, :]
    cos = torch.cat([ang.cos(), ang.cos()], -1).to(cs_dtype).cuda()
    sin = torch.cat([ang.sin(), ang.sin()], -1).to(cs_dtype).cuda()
    bs, nb = 16, M + 5
    k_pool = torch.zeros(nb, bs, H_kv, D, dtype=dtype, device="cuda")
    v_pool = torch.zeros_like(k_pool)
    dest_block = torch.randperm(nb, generator=g)[:M].cuda()
    dest_within = torch.randint(0, bs, (M,), generator=g).cuda()
    off = ops.pool_slot_offsets(dest_block, dest_within, k_pool)
    q = ops.rope_kv_write(qkv, H, H_kv, D, cos, sin, k_pool, v_pool, off)
    torch.cuda.synchronize()
    assert q.dtype == dtype
    x = qkv.float().view(M, H + 2 * H_kv, D)
    qr = _rope_ref(x[:, :H], cos.float(), sin.float())
    kr = _rope_ref(x[:, H:H + H_kv], cos.float(), sin.float())
    torch.testing.assert_close(q.float(), qr.transpose(0, 1).contiguous(), rtol=8e-3, atol=1e-2)
    torch.testing.assert_close(k_pool[dest_block, dest_within].float(), kr, rtol=8e-3, atol=1e-2)
    assert torch.equal(v_pool[dest_block, dest_within], qkv.view(M, H + 2 * H_kv, D)[:, H + H_kv:])
    untouched = torch.ones(nb, bs, dtype=torch.bool, device="cuda")
    untouched[dest_block, dest_within] = False
    assert torch.all(k_pool[untouched] == 0) and torch.all(v_pool[untouched] == 0)


@pytest.mark.parametrize("M,N,dtype", [(1, 4096, torch.bfloat16), (64, 4096, torch.bfloat16), (5, 8192, torch.bfloat16),
                                       (3, 136, torch.bfloat16), (64, 4096, torch.float16), (7, 1024, torch.float16)])
def test_rms_norm_matches_torch(M, N, dtype):
    g = torch.Generator().manual_seed(M + N)
    x = (torch.randn(M, N, generator=g) * 3).to(dtype).cuda()
    w = (torch.rand(N, generator=g) + 0.5).to(dtype).cuda()
    y = ops.rms_norm(x, w, 1e-5)
    xf = x.double()
    ref = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-5) * w.double()
    torch.testing.assert_close(y.double(), ref, rtol=8e-3, atol=1e-3)
    # transformers' own module (the engine's input/post-attention norms), same roundings: only
    # the fp32 reduction order of the mean differs
    from transformers.models.llama.modeling_llama import LlamaRMSNorm

    norm = LlamaRMSNorm(N, eps=1e-5).cuda().to(dtype)
    with torch.no_grad():
        norm.weight.copy_(w)
        tf = norm(x)
    assert y.dtype == dtype
    torch.testing.assert_close(y.float(), tf.float(), rtol=2 ** -7, atol=1e-3)
    assert (y == tf).float().mean().item() > 0.99


def test_one_workspace_serves_changing_shapes():
    """Small batches split positions over CTAs and use the workspace's arrival counters; calls
    of different shapes on one stream share one buffer, interleaved, and stay exact."""
    cases = [_case(E, 8, 2, 64, 16, [700] * E, seed=40 + E) for E in (1, 3, 2)]
    refs = []
    for q, kp, vp, bt, cl, mc in cases:
        refs.append(ref_paged_decode_attention(q.float().numpy(), kp.float().numpy(), vp.float().numpy(),
                                               bt.numpy(), cl.numpy()))
    for _ in range(2):
        for (q, kp, vp, bt, cl, mc), ref in zip(cases, refs):
            o = _run(q, kp, vp, bt, cl, mc)
            torch.cuda.synchronize()
            check_parity(o.reshape(-1, o.shape[-1]), ref.reshape(-1, ref.shape[-1]), "interleaved shapes")
    assert ops.device_status() == 0


@pytest.mark.parametrize("E,ctx", [(1, [1025]), (4, [1, 17, 300, 1024])])
def test_unsplit_launch_without_workspace(E, ctx):
    """split=False (no workspace: what the engine binding uses inside its graphs) gives the
    oracle's result too, for batches the planner would otherwise split."""
    q, k_pool, v_pool, bt, cl, max_ctx = _case(E, 32, 8, 128, 16, ctx, seed=5 + E)
    o = ops.paged_decode_attention(q.cuda(), k_pool.cuda(), v_pool.cuda(), bt.cuda(), cl.cuda(), max_ctx, split=False)
    torch.cuda.synchronize()
    ref = ref_paged_decode_attention(q.float().numpy(), k_pool.float().numpy(), v_pool.float().numpy(),
                                     bt.numpy(), cl.numpy())
    check_parity(o.reshape(E * 32, 128), ref.reshape(E * 32, 128), f"unsplit attention E={E}")
    assert ops.device_status() == 0


def test_unsplit_launch_with_the_engines_wide_block_table():
    """The engine's decode graphs size the launch by the block table's width (every block a
    sequence may ever hold: here 4096 blocks, max_context 65536 positions), far beyond the
    1024 block ids one CTA stages; the actual contexts are short.  The unsplit launch gives the
    oracle's result, and a context past the staged 1024 blocks is cut and reported
    (LSE_ERR_UNSUPPORTED on the status word), never read."""
    E, H, H_kv, D, bs = 3, 32, 8, 128, 16
    q, k_pool, v_pool, bt, cl, _ = _case(E, H, H_kv, D, bs, [5, 1000, 2049], seed=31)
    wide = torch.zeros(E, 4096, dtype=torch.int32)
    wide[:, : bt.shape[1]] = bt
    o = ops.paged_decode_attention(q.cuda(), k_pool.cuda(), v_pool.cuda(), wide.cuda(), cl.cuda(), 4096 * bs,
                                   split=False)
    torch.cuda.synchronize()
    ref = ref_paged_decode_attention(q.float().numpy(), k_pool.float().numpy(), v_pool.float().numpy(),
                                     bt.numpy(), cl.numpy())
    check_parity(o.reshape(E * H, D), ref.reshape(E * H, D), "unsplit attention, wide block table")
    assert ops.device_status() == 0
    # one sequence of 1025 blocks: cut at 1024 blocks and reported
    q, k_pool, v_pool, bt, cl, _ = _case(1, H, H_kv, D, bs, [1024 * bs + 3], seed=32)
    ops.paged_decode_attention(q.cuda(), k_pool.cuda(), v_pool.cuda(), bt.cuda(), cl.cuda(), 1024 * bs + 3,
                               split=False)
    assert ops.device_status() == _lib.LSE_ERR_UNSUPPORTED
    assert ops.device_status() == 0


@pytest.mark.parametrize("E,ctx,split", [(4, [1, 17, 300, 1024], True), (64, list(range(962, 1026)), True),
                                         (3, [5, 129, 2049], False)])
def test_paged_decode_attention_fp16(E, ctx, split):
    """fp16 q and pools (the reference's default dtype) on the fp16 MMA, split and unsplit,
    against the fp64 oracle on the same (fp16-rounded) inputs."""
    q, k_pool, v_pool, bt, cl, max_ctx = _case(E, 32, 8, 128, 16, ctx, seed=21 + E)
    q, k_pool, v_pool = q.half(), k_pool.half(), v_pool.half()
    o = ops.paged_decode_attention(q.cuda(), k_pool.cuda(), v_pool.cuda(), bt.cuda(), cl.cuda(), max_ctx, split=split)
    torch.cuda.synchronize()
    assert o.dtype == torch.float16
    ref = ref_paged_decode_attention(q.float().numpy(), k_pool.float().numpy(), v_pool.float().numpy(),
                                     bt.numpy(), cl.numpy())
    check_parity(o.reshape(E * 32, 128), ref.reshape(E * 32, 128), f"fp16 decode attention E={E}")
    assert ops.device_status() == 0
