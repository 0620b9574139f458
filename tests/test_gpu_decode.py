"""The end-to-end decode harness (llm_serving_engine_b200.llama_decode) at a small shape:
int8 projections against bf16 projections on the dequantized int8 weights, and the CUDA
graph of a decode step against the eager step."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from llm_serving_engine_b200.llama_decode import DecodeModel, LlamaShape, decode_bytes_per_step

pytestmark = pytest.mark.gpu

TINY = LlamaShape(layers=2, hidden=256, heads=4, kv_heads=2, head_dim=64, intermediate=512, vocab=1000)


@pytest.mark.parametrize("batch", [4, 24])  # fused gate_up + SiLU * mul kernel / tensor-core projection
def test_int8_step_matches_dequantized_bf16_step(batch):
    base = DecodeModel(TINY, batch=batch, context=16, device="cuda", seed=3, quantize=False)
    q8 = DecodeModel(TINY, batch=batch, context=16, device="cuda", seed=3, quantize=True, weights=base.weights)
    deq = q8.dequantized_weights(torch.bfloat16)
    ref = DecodeModel(TINY, batch=batch, context=16, device="cuda", seed=3, quantize=False, weights=deq)
    tokens = (torch.arange(batch, device="cuda") * 37) % TINY.vocab
    a, b = q8.logits(tokens), ref.logits(tokens)
    err = ((a - b).abs().max() / b.abs().max()).item()
    assert np.isfinite(err) and err < 2e-2, err


@pytest.mark.parametrize("batch", [16, 64])  # decode kernel / tensor-core kernel, as in config 4's step
def test_llama3_8b_int8_projections_on_live_activations(batch):
    """Config 4's model at full size (Llama-3-8B shape, 32 layers, paged attention over a
    1024-position context): every int8 projection of one decode step (fused QKV, o_proj, and
    the MLP's fused gate_up + SiLU * mul + down) is checked, on the activations it really
    receives in that step, against the fp32 product with its dequantized weights, at the
    kernels' parity tolerance (normwise 1e-2).  End to end, the step's logits agree with the
    same step run on bf16 projections of the dequantized weights within 1e-1 (32 random-init
    layers compound the two models' bf16 rounding differences)."""
    import torch.nn.functional as F

    from llm_serving_engine_b200.llama_decode import LLAMA3_8B

    q8 = DecodeModel(LLAMA3_8B, batch=batch, context=1024, device="cuda", seed=11, quantize=True)
    seen = []

    def recording(li, name, fn):
        def call(x, residual=None):
            seen.append((li, name, x.clone()))
            return fn(x) if residual is None else fn(x, residual=residual)
        return call

    orig = q8.proj
    q8.proj = [(recording(li, "qkv", qkv), recording(li, "o", o), recording(li, "mlp", mlp))
               for li, (qkv, o, mlp) in enumerate(orig)]
    tokens = (torch.arange(batch, device="cuda") * 1999) % LLAMA3_8B.vocab
    a = q8.logits(tokens)
    q8.proj = orig
    assert len(seen) == 3 * LLAMA3_8B.layers
    for li, name, x in seen:
        qkv, o, mlp = orig[li]
        xf = x.float()
        if name == "mlp":
            y = mlp(x).float()
            g = xf @ mlp.gate_weight().T
            ref = (F.silu(g) * (xf @ mlp.up_weight().T)) @ mlp.down_proj.dequantized(torch.float32).T
        else:
            mod = qkv if name == "qkv" else o
            y = mod(x).float()
            ref = xf @ mod.dequantized(torch.float32).T
        err = ((y - ref).abs().max() / ref.abs().max()).item()
        assert np.isfinite(err) and err <= 1e-2, f"layer {li} {name}: normwise {err:.3e}"
    deq = q8.dequantized_weights(torch.bfloat16)
    ref_model = DecodeModel(LLAMA3_8B, batch=batch, context=1024, device="cuda", seed=11, quantize=False,
                            weights=deq, kv=q8.kv)
    b = ref_model.logits(tokens)
    e2e = ((a - b).abs().max() / b.abs().max()).item()
    assert np.isfinite(e2e) and e2e < 1e-1, f"logits after 32 layers: normwise {e2e:.3e}"
    del q8, ref_model, deq, seen
    torch.cuda.empty_cache()


def test_graph_replay_equals_eager_step():
    m = DecodeModel(TINY, batch=8, context=32, device="cuda", seed=5, quantize=True)
    m.tokens.copy_(torch.arange(8, device="cuda") * 11)
    eager = m.step().clone()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        m.step()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=side):
        out = m.step()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)


def test_bytes_per_step_counts_int8_weights():
    assert decode_bytes_per_step(TINY, 4, 16, True) < decode_bytes_per_step(TINY, 4, 16, False)


def test_int8_lm_head_matches_dequantized_head():
    m = DecodeModel(TINY, batch=4, context=16, device="cuda", seed=7, quantize=True)
    tokens = torch.tensor([3, 5, 8, 13], device="cuda")
    bf = m.logits(tokens)
    m.set_lm_head_int8(True)
    q = m.logits(tokens)
    deq = m.lm_head_int8.dequantized(torch.float32)
    h = m._hidden(tokens, in_place=False).float()
    ref = h @ deq.T
    assert ((q - ref).abs().max() / ref.abs().max()).item() < 1e-2
    assert ((q - bf).abs().max() / bf.abs().max()).item() < 5e-2
    assert decode_bytes_per_step(TINY, 4, 16, True, int8_lm_head=True) < decode_bytes_per_step(TINY, 4, 16, True)


def test_paged_attention_step_matches_sdpa_on_the_same_cache():
    """The decode step with the paged kernel over a shuffled pool equals the step with torch
    SDPA over the same K/V laid out contiguously."""
    paged = DecodeModel(TINY, batch=5, context=37, device="cuda", seed=13, quantize=True, attention="paged")
    sdpa = DecodeModel(TINY, batch=5, context=37, device="cuda", seed=13, quantize=True, attention="sdpa",
                       weights=paged.weights)
    sdpa.proj = paged.proj
    bs, bt = paged.block_size, paged.kv["block_table"].long()
    pos = torch.arange(38, device="cuda")
    for li in range(TINY.layers):
        for name in ("k", "v"):
            pool = paged.kv[name][li]  # [nb, bs, Hkv, hd]
            gathered = pool[bt[:, pos // bs], pos % bs]  # [B, ctx + 1, Hkv, hd]
            sdpa.kv[name][li].copy_(gathered.permute(0, 2, 1, 3))
    tokens = torch.tensor([1, 2, 3, 500, 999], device="cuda")
    a, b = paged.logits(tokens), sdpa.logits(tokens)
    err = ((a - b).abs().max() / b.abs().max()).item()
    assert err < 2e-2, err


@pytest.mark.parametrize("batch", [4, 24])  # decode kernel / tensor-core kernel
def test_fused_norm_projections_give_the_same_step(batch):
    """fuse_norms=True (each RMSNorm fused into the projection that consumes it) produces the
    same logits bit for bit as the separate RMSNorm and projection launches."""
    m = DecodeModel(TINY, batch=batch, context=16, device="cuda", seed=9, quantize=True)
    tokens = (torch.arange(batch, device="cuda") * 13) % TINY.vocab
    separate = m.logits(tokens).clone()
    m.fuse_norms = True
    fused = m.logits(tokens)
    assert torch.equal(fused, separate)
