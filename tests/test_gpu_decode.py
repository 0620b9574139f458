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
def test_llama3_8b_int8_layers_match_dequantized_twin(batch):
    """Config 4's model at full size (Llama-3-8B shape, 32 layers, paged attention over a
    1024-position context), layer by layer: every layer of the int8 model and of its twin with
    bf16 projections on the dequantized int8 weights runs on the same input (the int8 model's
    own residual stream at that layer), and the two residual updates agree within normwise
    2e-2.  End to end, the logits after 32 random-init layers, where the two models' rounding
    differences compound, agree within 1e-1."""
    from llm_serving_engine_b200.llama_decode import LLAMA3_8B

    q8 = DecodeModel(LLAMA3_8B, batch=batch, context=1024, device="cuda", seed=11, quantize=True)
    deq = q8.dequantized_weights(torch.bfloat16)
    ref = DecodeModel(LLAMA3_8B, batch=batch, context=1024, device="cuda", seed=11, quantize=False, weights=deq,
                      kv=q8.kv)
    tokens = (torch.arange(batch, device="cuda") * 1999) % LLAMA3_8B.vocab
    trace: list = []
    a = q8._head(q8._hidden(tokens, in_place=False, trace=trace)).float()
    worst = 0.0
    for li, h in enumerate(trace):
        da = (q8.layer(li, h) - h).float()
        db = (ref.layer(li, h) - h).float()
        err = ((da - db).abs().max() / db.abs().max()).item()
        assert np.isfinite(err) and err < 2e-2, f"layer {li}: residual update normwise {err:.3e}"
        worst = max(worst, err)
    b = ref.logits(tokens)
    e2e = ((a - b).abs().max() / b.abs().max()).item()
    assert np.isfinite(e2e) and e2e < 1e-1, f"logits after 32 layers: normwise {e2e:.3e} (worst layer {worst:.3e})"
    del q8, ref, deq, trace
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
