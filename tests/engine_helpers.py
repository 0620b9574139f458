"""Helpers for the tests that drive the reference engine (`llm_serving_engine`, installed in
baseline/_ref) with the int8 modules: an int8-friendly tiny Llama checkpoint, sequences in
the states the reference scheduler leaves them in, and a forward that also returns logits.

The sequence bookkeeping follows what the reference's `scheduler_step` does for a prefill
chunk and a decode step (`src/llm_serving_engine/scheduling/scheduler.py`), as its own test
factories do (`tests/factories.py:38-48` of the reference).
"""

from __future__ import annotations

import copy

import pytest
import torch

ref = pytest.importorskip("llm_serving_engine", reason="the reference engine is not installed in baseline/_ref")

from llm_serving_engine.config import ModelConfig  # noqa: E402
from llm_serving_engine.model.model_runner import ModelRunner  # noqa: E402
from llm_serving_engine.model.sampling import SamplingParams  # noqa: E402
from llm_serving_engine.observability.metrics import RequestMetrics  # noqa: E402
from llm_serving_engine.scheduling.batch_plan import BatchEntry, BatchPlan  # noqa: E402
from llm_serving_engine.scheduling.sequence import Sequence  # noqa: E402

# hidden 256, 4 query heads of 64, 2 KV heads, MLP 512: every projection's K is a multiple of
# 16 and the fused QKV (N = 512) and gate_up (2 x 512) stay tile-friendly.
TINY = dict(vocab_size=128, hidden_size=256, intermediate_size=512, num_hidden_layers=2, num_attention_heads=4,
            num_key_value_heads=2, max_position_embeddings=512)


def save_tiny_llama(path, lm_head_gain: float = 30.0) -> str:
    """A random-init Llama-3-style checkpoint (seed 0) at `path`, bf16 on disk.  The lm_head is
    scaled by `lm_head_gain` so that the greedy token has a clear margin over the runner-up and
    an argmax comparison tests the projections, not rounding ties."""
    from transformers import LlamaConfig, LlamaForCausalLM

    torch.manual_seed(0)
    cfg = LlamaConfig(**TINY, bos_token_id=None, eos_token_id=None, pad_token_id=None, tie_word_embeddings=False)
    model = LlamaForCausalLM(cfg)
    with torch.no_grad():
        model.lm_head.weight.mul_(lm_head_gain)
    model.to(torch.bfloat16).save_pretrained(path)
    return str(path)


def load_runner(path, quantize: str = "none", dtype: str = "bfloat16", **overrides) -> ModelRunner:
    return ModelRunner(ModelConfig(model_name_or_path=str(path), device="cuda", dtype=dtype, quantize=quantize,
                                   **overrides))


def greedy_sequence(seq_id: int, prompt: list[int], max_tokens: int = 64) -> Sequence:
    return Sequence(seq_id=seq_id, prompt_tokens=list(prompt),
                    sampling_params=SamplingParams(temperature=0.0, max_tokens=max_tokens),
                    metrics=RequestMetrics(enqueue_time=0.0))


def prefill_entry(seq: Sequence, n_tokens: int) -> BatchEntry:
    """The scheduler's bookkeeping for one prefill chunk of `seq`."""
    seq.prefill_progress += n_tokens
    seq.status = "DECODING" if seq.prefill_progress == seq.num_tokens else "PREFILLING"
    return BatchEntry(seq.seq_id, n_tokens, is_prefill_chunk=True)


def decode_plan(seqs) -> BatchPlan:
    return BatchPlan(entries=[BatchEntry(seq.seq_id, 1, is_prefill_chunk=False) for seq in seqs])


def forward_fused_with_logits(runner: ModelRunner, plan: BatchPlan, seqs: dict):
    """`runner.forward_fused(plan, seqs)` and the logits it sampled from (float32)."""
    seen = {}
    original = runner.emit_tokens

    def grab(logits, owed):
        seen["logits"] = logits[: len(owed)].float().clone()
        return original(logits, owed)

    runner.emit_tokens = grab
    try:
        out = runner.forward_fused(plan, seqs)
    finally:
        del runner.emit_tokens
    return out, seen.get("logits")


def prefilled(runner: ModelRunner, allocator, seq_id: int, prompt: list[int]) -> Sequence:
    """A sequence whose prompt went through one prefill (forward_fused), with its first token
    generated and a KV slot allocated for the next decode step."""
    seq = greedy_sequence(seq_id, prompt)
    assert allocator.allocate(seq, len(prompt))
    [(_, token, _)] = runner.forward_fused(BatchPlan(entries=[prefill_entry(seq, len(prompt))]), {seq_id: seq})
    seq.generated_tokens.append(token)
    assert allocator.allocate(seq, 1)
    return seq


def advance(allocator, seqs: list, results: list) -> None:
    by_id = {seq.seq_id: seq for seq in seqs}
    for seq_id, token, _finished in results:
        by_id[seq_id].generated_tokens.append(token)
        assert allocator.allocate(by_id[seq_id], 1)


def eager_then(runner: ModelRunner, plan: BatchPlan, seqs: dict, monkeypatch):
    """(eager forward_fused results on a copy of `seqs`, runner.forward results) with
    forward_fused disabled for the second call, so that it can only have replayed a graph."""
    eager = runner.forward_fused(plan, copy.deepcopy(seqs))

    def refuse(*args, **kwargs):
        raise AssertionError("the plan ran eagerly instead of replaying a graph")

    with monkeypatch.context() as patch:
        patch.setattr(runner, "forward_fused", refuse)
        graphed = runner.forward(plan, seqs)
    return eager, graphed
