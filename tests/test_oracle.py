"""The CPU oracle, pinned before anything is checked against it (CPU only)."""

from __future__ import annotations

import hashlib
import os

import numpy as np
import pytest
import torch

from llm_serving_engine_b200.inputs import make_inputs
from oracle import clib
from oracle.ref_linear import (
    bf16_bits_to_f32,
    f32_to_bf16_bits,
    parity_errors,
    ref_fused_split,
    ref_int8_linear,
    ref_mlp,
    ref_quantize,
)

PROJ = ("q_proj", "k_proj", "v_proj", "o_proj")


@pytest.fixture(scope="module")
def tiny(golden_dir):
    return dict(np.load(os.path.join(golden_dir, "ref_tiny_llama_int8.npz")))


# ---- pinned against the reference's own CPU path ---------------------------------------

@pytest.mark.parametrize("layer", [0, 1])
@pytest.mark.parametrize("proj", PROJ)
def test_oracle_reproduces_reference_projection(tiny, layer, proj):
    """Each q/k/v/o output the reference's `_forward_hf` computed with nn.Linear on the
    dequantized weight equals the oracle on the recorded input."""
    p = f"l{layer}.{proj}"
    ref = ref_int8_linear(tiny[f"{p}.x"], tiny[f"{p}.q"], tiny[f"{p}.s"])
    np.testing.assert_allclose(ref, tiny[f"{p}.y"], rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("layer", [0, 1])
def test_oracle_mlp_matches_reference(tiny, layer):
    """`layer.mlp(x)` of the reference (down(silu(gate) * up)) equals the oracle MLP."""
    p = f"l{layer}"
    ref = ref_mlp(tiny[f"{p}.mlp.x"],
                  tiny[f"{p}.gate_proj.q"], tiny[f"{p}.gate_proj.s"],
                  tiny[f"{p}.up_proj.q"], tiny[f"{p}.up_proj.s"],
                  tiny[f"{p}.down_proj.q"], tiny[f"{p}.down_proj.s"])
    np.testing.assert_allclose(ref, tiny[f"{p}.mlp.y"], rtol=1e-4, atol=1e-6)


@pytest.mark.parametrize("layer", [0, 1])
def test_fused_qkv_split_matches_separate_projections(tiny, layer):
    """A fused [q; k; v] weight split by columns reproduces the three reference outputs."""
    p = f"l{layer}"
    x = tiny[f"{p}.q_proj.x"]
    q = np.concatenate([tiny[f"{p}.{n}.q"] for n in ("q_proj", "k_proj", "v_proj")])
    s = np.concatenate([tiny[f"{p}.{n}.s"] for n in ("q_proj", "k_proj", "v_proj")])
    sizes = [tiny[f"{p}.{n}.q"].shape[0] for n in ("q_proj", "k_proj", "v_proj")]
    parts = ref_fused_split(ref_int8_linear(x, q, s), sizes)
    for part, n in zip(parts, ("q_proj", "k_proj", "v_proj")):
        np.testing.assert_allclose(part, tiny[f"{p}.{n}.y"], rtol=1e-5, atol=1e-6)


def test_config1_inputs_and_outputs_reproduce(golden_dir):
    """Config 1, the CPU case (M=8, K=2048, N=2048): the seeded generator gives the recorded
    bits, the oracle gives the recorded output, and it agrees with the reference's CPU
    nn.Linear."""
    g = np.load(os.path.join(golden_dir, "config1.npz"))
    x, w, s = make_inputs(8, 2048, 2048, seed=0)
    sha = lambda t: hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()  # noqa: E731
    assert sha(x) == str(g["sha_x"]) and sha(w) == str(g["sha_w"]) and sha(s) == str(g["sha_s"])
    y = ref_int8_linear(x.float().numpy(), w.numpy(), s.numpy())
    np.testing.assert_allclose(y, g["y_oracle"], rtol=1e-6, atol=1e-7)
    nw, ok, _ = parity_errors(g["y_ref_cpu"], y)
    assert nw < 1e-5 and ok


# ---- the C restatement agrees with the numpy one ---------------------------------------

@pytest.mark.parametrize("M,K,N", [(1, 16, 8), (3, 48, 17), (8, 256, 64), (5, 1024, 33)])
def test_c_oracle_matches_numpy(M, K, N):
    rng = np.random.default_rng(M * 1000 + K + N)
    x = rng.standard_normal((M, K)).astype(np.float32)
    q = rng.integers(-127, 128, (N, K), dtype=np.int8)
    s = rng.uniform(1e-4, 5e-4, N).astype(np.float32)
    np.testing.assert_allclose(clib.c_int8_linear(x, q, s), ref_int8_linear(x, q, s), rtol=1e-12, atol=1e-15)


@pytest.mark.parametrize("N,K", [(4, 16), (33, 100), (64, 2048)])
def test_c_quantizer_bit_exact_with_numpy(N, K):
    rng = np.random.default_rng(N + K)
    w = (rng.standard_normal((N, K)) * rng.uniform(0.01, 3, (N, 1))).astype(np.float32)
    w[0, :] = 0.0  # an all-zero row
    qn, sn = ref_quantize(w)
    qc, sc = clib.c_quantize(w)
    assert np.array_equal(qn, qc)
    assert np.array_equal(sn.view(np.uint32), sc.view(np.uint32))


# ---- known-answer tests ------------------------------------------------------------------

def test_known_answer_identity_like():
    K = N = 32
    q = np.eye(N, K, dtype=np.int8) * 127
    s = np.full(N, 1 / 127, dtype=np.float32)
    x = np.arange(2 * K, dtype=np.float32).reshape(2, K)
    np.testing.assert_allclose(ref_int8_linear(x, q, s), x * (127 * np.float64(np.float32(1 / 127))), rtol=1e-12)


def test_known_answer_single_nonzero_column():
    q = np.zeros((5, 16), dtype=np.int8)
    q[:, 7] = np.array([1, -1, 127, -127, 3], dtype=np.int8)
    s = np.array([1, 2, 0.5, 0.25, 1e-4], dtype=np.float32)
    x = np.zeros((2, 16), dtype=np.float32)
    x[0, 7], x[1, 7] = 2.0, -3.0
    y = ref_int8_linear(x, q, s)
    expect = np.outer([2.0, -3.0], q[:, 7].astype(np.float64) * s.astype(np.float64))
    np.testing.assert_array_equal(y, expect)


def test_known_answer_extremes():
    """All-+127 / all--127 weights: y = +-127 * s * sum(x)."""
    K = 4096
    q = np.stack([np.full(K, 127, np.int8), np.full(K, -127, np.int8)])
    s = np.array([5e-4, 1e-4], dtype=np.float32)
    x = np.ones((1, K), dtype=np.float32)
    np.testing.assert_allclose(ref_int8_linear(x, q, s)[0], [127 * K * np.float64(s[0]), -127 * K * np.float64(s[1])])


def test_quantizer_properties():
    rng = np.random.default_rng(0)
    w = rng.standard_normal((16, 64)).astype(np.float32)
    w[3] = 0.0
    q, s = ref_quantize(w)
    assert q.dtype == np.int8 and np.all(np.abs(q.astype(np.int32)) <= 127)
    assert s[3] == 1.0 and np.all(q[3] == 0)
    # the channel max maps to +-127 exactly, and dequantization error is at most s/2
    assert np.all(np.max(np.abs(q[np.arange(16) != 3].astype(np.int32)), axis=1) == 127)
    err = np.abs(q.astype(np.float64) * s[:, None] - w)
    assert np.all(err <= s[:, None] / 2 * (1 + 1e-6))


def test_bf16_round_trip():
    x = np.array([1.0, -2.5, 3.14159, 1e-3, 65504.0, -0.0], dtype=np.float32)
    bits = f32_to_bf16_bits(x)
    back = bf16_bits_to_f32(bits)
    ref = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    np.testing.assert_array_equal(back, ref)


def test_parity_metric_definition():
    ref = np.array([[1.0, -2.0, 0.0, 4.0]])
    y = ref + np.array([[0.005, 0.0, 0.002, -0.03]])
    nw, ok, ratio = parity_errors(y, ref)
    assert nw == pytest.approx(0.03 / 4)
    assert ok and ratio <= 1
    nw, ok, _ = parity_errors(ref + np.array([[0.0, 0.0, 0.0, 0.1]]), ref)
    assert not ok and nw == pytest.approx(0.025)
    # a planted mistake in the oracle (one wrong sign) is caught by the criterion
    q = np.ones((4, 16), np.int8)
    s = np.ones(4, np.float32)
    x = np.ones((2, 16), np.float32)
    good = ref_int8_linear(x, q, s)
    bad = good.copy()
    bad[1, 2] = -bad[1, 2]
    assert not parity_errors(bad, good)[1]


def test_attention_oracle_matches_torch_sdpa_in_float64():
    """Pin the paged decode-attention oracle: gathered through a shuffled block table, it
    equals torch's scaled_dot_product_attention (float64, GQA) on the contiguous K/V."""
    import torch
    import torch.nn.functional as F

    from oracle.ref_attention import gather_kv, ref_paged_decode_attention

    g = torch.Generator().manual_seed(0)
    E, H, H_kv, D, bs = 3, 8, 2, 16, 4
    ctx = np.array([1, 9, 13])
    nbps = 4
    bt = torch.randperm(E * nbps + 2, generator=g)[: E * nbps].view(E, nbps).numpy()
    k_pool = torch.randn(E * nbps + 2, bs, H_kv, D, generator=g, dtype=torch.float64).numpy()
    v_pool = torch.randn(E * nbps + 2, bs, H_kv, D, generator=g, dtype=torch.float64).numpy()
    q = torch.randn(E, H, D, generator=g, dtype=torch.float64).numpy()
    out = ref_paged_decode_attention(q, k_pool, v_pool, bt, ctx)
    for e in range(E):
        k = torch.from_numpy(gather_kv(k_pool, bt, e, int(ctx[e]))).permute(1, 0, 2)[None]
        v = torch.from_numpy(gather_kv(v_pool, bt, e, int(ctx[e]))).permute(1, 0, 2)[None]
        ref = F.scaled_dot_product_attention(torch.from_numpy(q[e])[None, :, None], k, v, enable_gqa=True)
        np.testing.assert_allclose(out[e], ref[0, :, 0].numpy(), rtol=1e-12, atol=1e-12)
    assert np.all(ref_paged_decode_attention(q, k_pool, v_pool, bt, np.array([0, 0, 0])) == 0)


def test_multi_token_attention_oracle_matches_torch_sdpa_and_the_decode_oracle():
    """Pin the multi-token paged-attention oracle (`paged_attention_2`'s general case): entries
    with chunks of several tokens after a cached prefix equal torch's causal SDPA (float64,
    GQA) over the contiguous K/V with the queries placed at their positions; single-token
    entries at query_offset = context_len - 1 equal the decode oracle; rows of no entry stay
    zero."""
    import torch
    import torch.nn.functional as F

    from oracle.ref_attention import gather_kv, ref_paged_attention, ref_paged_decode_attention

    g = torch.Generator().manual_seed(1)
    H, H_kv, D, bs = 8, 2, 16, 4
    q_len = np.array([5, 1, 3, 1])
    query_offset = np.array([0, 6, 9, 0])           # a fresh prefill, decodes, a chunk after a prefix
    context_len = query_offset + q_len
    q_start = np.concatenate([[0], np.cumsum(q_len)[:-1]]) + 1  # row 0 belongs to no entry
    T = int(q_start[-1] + q_len[-1]) + 2
    E, nbps = len(q_len), 4
    bt = torch.randperm(E * nbps + 2, generator=g)[: E * nbps].view(E, nbps).numpy()
    k_pool = torch.randn(E * nbps + 2, bs, H_kv, D, generator=g, dtype=torch.float64).numpy()
    v_pool = torch.randn(E * nbps + 2, bs, H_kv, D, generator=g, dtype=torch.float64).numpy()
    q = torch.randn(H, T, D, generator=g, dtype=torch.float64).numpy()
    out = ref_paged_attention(q, k_pool, v_pool, bt, context_len, query_offset, q_start, q_len)
    for e in range(E):
        ctx, off, qs, ql = int(context_len[e]), int(query_offset[e]), int(q_start[e]), int(q_len[e])
        k = torch.from_numpy(gather_kv(k_pool, bt, e, ctx)).permute(1, 0, 2)[None]
        v = torch.from_numpy(gather_kv(v_pool, bt, e, ctx)).permute(1, 0, 2)[None]
        qe = torch.from_numpy(q[:, qs:qs + ql])[None]
        mask = torch.arange(ctx)[None, :] <= (off + torch.arange(ql))[:, None]
        ref = F.scaled_dot_product_attention(qe, k, v, attn_mask=mask, enable_gqa=True)
        np.testing.assert_allclose(out[:, qs:qs + ql], ref[0].numpy(), rtol=1e-12, atol=1e-12)
        if ql == 1:
            dec = ref_paged_decode_attention(q[:, qs].reshape(1, H, D), k_pool, v_pool, bt[e:e + 1], context_len[e:e + 1])
            np.testing.assert_allclose(out[:, qs], dec[0], rtol=1e-12, atol=1e-12)
    assert np.all(out[:, 0] == 0) and np.all(out[:, -2:] == 0)


def test_pack_layout_restatement_places_every_byte():
    """The packed layout's checker puts W[n, k] at (n // 16) * 16 * Kp + (k // 128) * 2048 +
    (n // 8 % 2) * 1024 + (k // 64 % 2) * 512 + (n % 8) * 64 + ((k // 16 % 4) ^ (n % 8 // 2)) * 16
    + k % 16, with zero padding to multiples of 128: the 64-byte-swizzled K-major atoms the
    tensor core reads as its operand and the decode kernel's fragments come from."""
    from oracle.ref_linear import ref_pack_weight

    rng = np.random.default_rng(5)
    for N, K in ((8, 16), (130, 200), (256, 384)):
        w = rng.integers(-127, 128, size=(N, K), dtype=np.int8)
        p = ref_pack_weight(w)
        Np, Kp = -(-N // 128) * 128, -(-K // 128) * 128
        assert p.shape == (Np * Kp,)
        n, k = np.meshgrid(np.arange(N), np.arange(K), indexing="ij")
        off = ((n // 16) * 16 * Kp + (k // 128) * 2048 + (n // 8 % 2) * 1024 + (k // 64 % 2) * 512 + (n % 8) * 64
               + (((k // 16) % 4) ^ ((n % 8) // 2)) * 16 + k % 16)
        assert np.array_equal(p[off], w)
        mask = np.ones(Np * Kp, dtype=bool)
        mask[off.ravel()] = False
        assert not p[mask].any()
