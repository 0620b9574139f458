"""The int8 modules inside the reference engine itself (GPU).

These run the reference's own code paths, unmodified, from its install in baseline/_ref, with
`ModelConfig(quantize="int8")` bound by `engine_hook.install()`:

* `ModelRunner.__init__` with `quantize="int8"` (`src/llm_serving_engine/model/model_runner.py:
  44-53`; the reference raises there and pins the raise in `tests/test_model_runner.py:120-122`:
  here the same call loads an int8 model);
* `forward_fused` (`model_runner.py:203-211`) against a twin runner whose projections are the
  dequantized int8 weights in bf16 (same greedy tokens, logits within tolerance);
* `DecodeGraphRunner.capture` / `_self_check` / `replay` (`decode_graph.py:87-140,214-226`):
  every bucket captured and kept (as `tests/test_decode_graph.py:28` asserts), replay == eager
  (`tests/test_decode_graph.py:53-59`);
* `PiecewiseGraphRunner.capture` / `_self_check` / `replay` (`piecewise_graph.py:71-183,
  222-235`): every bucket kept (`tests/test_piecewise_graph.py:28`), replay == eager
  (`tests/test_piecewise_graph.py:47-58`), on the decode kernel and both token tiles of the
  tensor-core kernel;
* `bytes_beyond_kv_pool` (`model_runner.py:131-159`), the engine's memory probe, including
  its eager dummy iteration at 4160 tokens;
* `decoder_hidden` (`model_runner.py:213-224`) with the residual adds in the o_proj and down
  epilogues, against the reference's own loop on the same int8 weights.

A failed `_self_check` makes the reference drop its graphs silently and run eagerly; the
assertions on the graph dicts and the refusal of `forward_fused` during replay make such a
fallback fail here.
"""

from __future__ import annotations

import pytest
import torch

from tests.engine_helpers import (BatchPlan, advance, decode_plan, eager_then, forward_fused_with_logits,
                                  greedy_sequence, load_runner, prefill_entry, prefilled, save_tiny_llama)

pytestmark = pytest.mark.gpu

from llm_serving_engine.model.decode_graph import decode_graph_buckets  # noqa: E402
from llm_serving_engine.model.piecewise_graph import piecewise_graph_buckets  # noqa: E402
from llm_serving_engine.scheduling.allocator import BlockAllocator  # noqa: E402

from llm_serving_engine_b200 import engine_hook  # noqa: E402
from llm_serving_engine_b200.int8_linear import FusedInt8QKV, Int8Linear, Int8LlamaMLP, _SliceOf  # noqa: E402

NUM_BLOCKS, BLOCK_SIZE = 96, 16


@pytest.fixture(scope="module")
def tiny_dir(tmp_path_factory):
    return save_tiny_llama(tmp_path_factory.mktemp("tiny-int8-llama"))


@pytest.fixture(scope="module", autouse=True)
def _hook():
    engine_hook.install()
    yield
    engine_hook.uninstall()


def _int8_runner(tiny_dir, dtype="bfloat16"):
    runner = load_runner(tiny_dir, quantize="int8", dtype=dtype)
    runner.allocate_kv_pool(NUM_BLOCKS, BLOCK_SIZE)
    return runner


def _twin_runner(tiny_dir, int8_runner, dtype="bfloat16"):
    """The same checkpoint with every projection replaced by the int8 runner's dequantized
    weights (in the model dtype), run by the reference's own path (cuBLAS nn.Linear, Triton
    attention)."""
    twin = load_runner(tiny_dir, quantize="none", dtype=dtype)
    with torch.no_grad():
        for lt, li in zip(twin._layers, int8_runner._layers, strict=True):
            qkv = li.self_attn.qkv_int8
            wq, wk, wv = torch.split(qkv.fused.dequantized(torch.float32), qkv.sizes, dim=0)
            lt.self_attn.q_proj.weight.copy_(wq)
            lt.self_attn.k_proj.weight.copy_(wk)
            lt.self_attn.v_proj.weight.copy_(wv)
            lt.self_attn.o_proj.weight.copy_(li.self_attn.o_proj.dequantized(torch.float32))
            lt.mlp.gate_proj.weight.copy_(li.mlp.gate_weight())
            lt.mlp.up_proj.weight.copy_(li.mlp.up_weight())
            lt.mlp.down_proj.weight.copy_(li.mlp.down_proj.dequantized(torch.float32))
    twin.allocate_kv_pool(NUM_BLOCKS, BLOCK_SIZE)
    return twin


def test_quantize_int8_config_loads_an_int8_model(tiny_dir):
    """The call the reference pins as NotImplementedError loads, with every projection slot
    holding an int8 module and the config still saying int8."""
    runner = load_runner(tiny_dir, quantize="int8")
    assert runner.config.quantize == "int8"
    assert runner.model.dtype == torch.bfloat16
    for layer in runner._layers:
        attn = layer.self_attn
        assert isinstance(attn.qkv_int8, FusedInt8QKV)
        assert all(isinstance(p, _SliceOf) for p in (attn.q_proj, attn.k_proj, attn.v_proj))
        assert isinstance(attn.o_proj, Int8Linear)
        assert isinstance(layer.mlp, Int8LlamaMLP)
    # the reference's own checks on the loaded model still pass (model_runner.py:77-94)
    runner.check_custom_kernel_support()


@pytest.mark.parametrize("dtype", ["bfloat16", "float16"])
@pytest.mark.parametrize("prompt_lens", [(5,), (3, 17, 40)])
def test_forward_fused_matches_dequantized_twin(tiny_dir, prompt_lens, dtype):
    """Prefill then two decode steps through the reference's eager forward_fused, in bf16 and in
    fp16 (the reference's default dtype, run natively by the int8 operators): the int8 runner
    and its dequantized twin give logits within normwise 2e-2 of the largest logit (16-bit
    activations through two layers) and the same greedy token wherever the twin's margin
    between its two best tokens exceeds four times the largest logit difference.  Both runners
    then continue with the twin's tokens, so one near-tie cannot make the sequences diverge."""
    runner = _int8_runner(tiny_dir, dtype)
    twin = _twin_runner(tiny_dir, runner, dtype)
    alloc_a, alloc_b = BlockAllocator(NUM_BLOCKS, BLOCK_SIZE), BlockAllocator(NUM_BLOCKS, BLOCK_SIZE)
    prompts = [[(7 * i + 3 * j) % 120 + 1 for j in range(n)] for i, n in enumerate(prompt_lens)]
    seqs_a = [greedy_sequence(100 + i, p) for i, p in enumerate(prompts)]
    seqs_b = [greedy_sequence(100 + i, p) for i, p in enumerate(prompts)]
    for sa, sb in zip(seqs_a, seqs_b, strict=True):
        assert alloc_a.allocate(sa, sa.num_tokens) and alloc_b.allocate(sb, sb.num_tokens)
    plan_a = BatchPlan(entries=[prefill_entry(s, s.num_tokens) for s in seqs_a])
    plan_b = BatchPlan(entries=[prefill_entry(s, s.num_tokens) for s in seqs_b])
    decisive = 0
    for step in range(3):
        out_a, logits_a = forward_fused_with_logits(runner, plan_a, {s.seq_id: s for s in seqs_a})
        out_b, logits_b = forward_fused_with_logits(twin, plan_b, {s.seq_id: s for s in seqs_b})
        diff = (logits_a - logits_b).abs()
        err = diff.max().item() / logits_b.abs().max().item()
        assert err <= 2e-2, f"step {step}: logits normwise {err:.3e}"
        top2 = logits_b.topk(2, dim=-1).values
        for row, ((ida, tok_a, _), (idb, tok_b, _)) in enumerate(zip(out_a, out_b, strict=True)):
            assert ida == idb
            if (top2[row, 0] - top2[row, 1]).item() > 4 * diff[row].max().item():
                decisive += 1
                assert tok_a == tok_b, f"step {step}, sequence {ida}: greedy token {tok_a} != twin's {tok_b}"
        advance(alloc_a, seqs_a, out_b)
        advance(alloc_b, seqs_b, out_b)
        plan_a, plan_b = decode_plan(seqs_a), decode_plan(seqs_b)
    assert decisive >= 2 * len(prompt_lens), f"only {decisive} decisive rows"


@pytest.mark.parametrize("dtype", ["bfloat16", "float16"])
def test_residual_adds_run_in_the_projection_epilogues(tiny_dir, dtype):
    """With the switch's defaults every layer's o_proj and MLP receive the layer's residual (the
    adds run in their kernels' epilogues) in prefill and decode; the logits agree with the
    reference's own layer loop on the same int8 weights (the bound methods removed) within the
    one rounding per add that the fused form saves, and the greedy tokens are the same
    wherever that loop's top-two margin exceeds four times the largest logit difference."""
    runner = _int8_runner(tiny_dir, dtype)
    plain = _int8_runner(tiny_dir, dtype)
    del plain.decoder_hidden, plain.attention_output  # back to the class's methods
    seen = []
    for layer in runner._layers:
        for mod in (layer.self_attn.o_proj, layer.mlp):
            inner = mod.forward
            mod.forward = (lambda f: lambda x, residual=None: seen.append(residual is not None) or f(x, residual))(inner)
    alloc_a, alloc_b = BlockAllocator(NUM_BLOCKS, BLOCK_SIZE), BlockAllocator(NUM_BLOCKS, BLOCK_SIZE)
    prompts = [[(5 * i + 2 * j) % 120 + 1 for j in range(n)] for i, n in enumerate((4, 21))]
    seqs_a = [greedy_sequence(400 + i, p) for i, p in enumerate(prompts)]
    seqs_b = [greedy_sequence(400 + i, p) for i, p in enumerate(prompts)]
    for sa, sb in zip(seqs_a, seqs_b, strict=True):
        assert alloc_a.allocate(sa, sa.num_tokens) and alloc_b.allocate(sb, sb.num_tokens)
    plan_a = BatchPlan(entries=[prefill_entry(s, s.num_tokens) for s in seqs_a])
    plan_b = BatchPlan(entries=[prefill_entry(s, s.num_tokens) for s in seqs_b])
    for step in range(3):
        seen.clear()
        out_a, logits_a = forward_fused_with_logits(runner, plan_a, {s.seq_id: s for s in seqs_a})
        out_b, logits_b = forward_fused_with_logits(plain, plan_b, {s.seq_id: s for s in seqs_b})
        assert seen == [True] * (2 * len(runner._layers)), f"step {step}: residuals not handed over: {seen}"
        diff = (logits_a - logits_b).abs()
        assert diff.max().item() <= 1e-2 * logits_b.abs().max().item(), f"step {step}"
        top2 = logits_b.topk(2, dim=-1).values
        for row, ((_, tok_a, _), (_, tok_b, _)) in enumerate(zip(out_a, out_b, strict=True)):
            if (top2[row, 0] - top2[row, 1]).item() > 4 * diff[row].max().item():
                assert tok_a == tok_b
        advance(alloc_a, seqs_a, out_b)
        advance(alloc_b, seqs_b, out_b)
        plan_a, plan_b = decode_plan(seqs_a), decode_plan(seqs_b)


@pytest.mark.parametrize("dtype", ["bfloat16", "float16"])
def test_decode_graphs_capture_self_check_and_replay_equal_eager(tiny_dir, monkeypatch, dtype):
    runner = _int8_runner(tiny_dir, dtype)
    buckets = decode_graph_buckets(8)
    runner.capture_decode_graphs(buckets)
    assert set(runner._decode_graphs.graphs) == set(buckets), "capture or self-check failed"
    alloc = BlockAllocator(NUM_BLOCKS, BLOCK_SIZE)
    seqs = [prefilled(runner, alloc, 200 + i, [(5 * i + j) % 120 + 1 for j in range(n)])
            for i, n in enumerate([3, 9, 20, 33, 6])]
    for batch in (seqs[:1], seqs[:3], seqs):  # buckets 1, 4 (one padding row), 8 (three)
        for _ in range(2):
            eager, graphed = eager_then(runner, decode_plan(batch), {s.seq_id: s for s in batch}, monkeypatch)
            assert graphed == eager
            advance(alloc, batch, graphed)


def test_piecewise_graphs_capture_self_check_and_replay_equal_eager(tiny_dir, monkeypatch):
    """Buckets 16 (the decode kernel), 24/48/64 (tensor-core kernel, 64-token tile) and 96
    (128-token tile): every one kept after the self-check, replay == eager on mixed plans."""
    runner = _int8_runner(tiny_dir)
    buckets = piecewise_graph_buckets(96)
    runner.capture_piecewise_graphs(buckets)
    assert set(runner._piecewise_graphs.graphs) == set(buckets), "capture or self-check failed"
    alloc = BlockAllocator(NUM_BLOCKS, BLOCK_SIZE)
    decoders = [prefilled(runner, alloc, 300 + i, [(3 * i + j) % 120 + 1 for j in range(n)])
                for i, n in enumerate([3, 7, 5])]
    # 3 decodes + 9 prefill tokens -> bucket 16, 4 + 14 -> 24, 5 + 40 -> 48, 6 + 80 -> 96
    for new_len, seq_id in ((9, 310), (14, 311), (40, 312), (80, 313)):
        newcomer = greedy_sequence(seq_id, [(j * 11 + seq_id) % 120 + 1 for j in range(new_len)])
        assert alloc.allocate(newcomer, new_len)
        plan = BatchPlan(entries=[*decode_plan(decoders).entries, prefill_entry(newcomer, new_len)])
        seqs = {s.seq_id: s for s in [*decoders, newcomer]}
        eager, graphed = eager_then(runner, plan, seqs, monkeypatch)
        assert graphed == eager
        advance(alloc, [*decoders, newcomer], graphed)
        decoders.append(newcomer)


def test_bytes_beyond_kv_pool_runs_the_int8_captures_and_dummy(tiny_dir):
    """The engine's start-up memory probe: captures (with self-checks) against a one-block pool
    and one eager 4160-token dummy iteration, all through the int8 kernels."""
    runner = load_runner(tiny_dir, quantize="int8")
    extra = runner.bytes_beyond_kv_pool(BLOCK_SIZE, 4160, decode_graph_buckets(4), [16, 24, 4160])
    assert extra > 0
    assert runner._k_pool is None  # the probe releases its pool and graphs
