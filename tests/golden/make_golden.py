"""Generate the golden fixtures under tests/golden/ (run once, in a container that has the
reference checked out; the fixtures are committed and the tests never import the reference).

    python tests/golden/make_golden.py /path/to/llm-serving-engine

Fixtures
--------
ref_tiny_llama_int8.npz
    The reference's own CPU forward path (`ModelRunner.forward` ->
    `ModelRunner._forward_hf`, `src/llm_serving_engine/model/model_runner.py:170-200`) run on
    a tiny random Llama whose projection weights were replaced by their int8 dequantization
    `q * s[:, None]` (q, s from the oracle quantizer).  Forward hooks record, for every
    decoder layer, the input and output of q_proj, k_proj, v_proj, o_proj (the `nn.Linear`
    calls at `model_runner.py:322-324` and the o_proj HF attention makes) and of the MLP
    (`layer.mlp`, `model_runner.py:223`), plus q/s of each projection and the reference's
    greedy token and last-row logits.  The oracle must reproduce every recorded output from
    the recorded input and (q, s): that pins the oracle to the reference's arithmetic at the
    boundary the int8 layer replaces.  The model config is the reference's own
    `tiny_llama_dir` fixture (`tests/conftest.py:24-39`: vocab 64, hidden 32, intermediate 64,
    2 layers, 4 heads, 2 KV heads, seed 0).

config1.npz
    Config 1, the CPU case (x bf16 [8, 2048] ~ N(0,1), W int8 [2048, 2048] uniform [-127, 127],
    s uniform [1e-4, 5e-4], seed 0): SHA-256 of the seeded inputs, the oracle output, and the
    output of the reference's CPU nn.Linear (float32 `F.linear` on the dequantized weight) on
    the same inputs.
"""

from __future__ import annotations

import hashlib
import os
import sys
import tempfile

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from llm_serving_engine_b200.inputs import make_inputs  # noqa: E402
from oracle.ref_linear import ref_int8_linear, ref_quantize  # noqa: E402

PROJ = ("q_proj", "k_proj", "v_proj", "o_proj")


def sha256(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


def tiny_llama_fixture(ref_root: str) -> None:
    sys.path.insert(0, os.path.join(ref_root, "src"))
    sys.path.insert(0, ref_root)
    from transformers import LlamaConfig, LlamaForCausalLM

    from llm_serving_engine.config import ModelConfig
    from llm_serving_engine.model.model_runner import ModelRunner
    from llm_serving_engine.model.sampling import SamplingParams
    from llm_serving_engine.observability.metrics import RequestMetrics
    from llm_serving_engine.scheduling.batch_plan import BatchEntry, BatchPlan
    from llm_serving_engine.scheduling.sequence import Sequence

    torch.manual_seed(0)
    config = LlamaConfig(
        vocab_size=64, hidden_size=32, intermediate_size=64, num_hidden_layers=2,
        num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=64,
        bos_token_id=None, eos_token_id=None, pad_token_id=None,
    )
    model = LlamaForCausalLM(config)
    out: dict[str, np.ndarray] = {}
    with torch.no_grad():
        for li, layer in enumerate(model.model.layers):
            mods = {p: getattr(layer.self_attn, p) for p in PROJ}
            mods.update({p: getattr(layer.mlp, p) for p in ("gate_proj", "up_proj", "down_proj")})
            for name, lin in mods.items():
                q, s = ref_quantize(lin.weight.float().numpy())
                out[f"l{li}.{name}.q"] = q
                out[f"l{li}.{name}.s"] = s
                lin.weight.copy_(torch.from_numpy(q.astype(np.float32) * s[:, None]))

    with tempfile.TemporaryDirectory() as tmp:
        model.save_pretrained(tmp)
        runner = ModelRunner(ModelConfig(model_name_or_path=tmp, device="cpu", dtype="float32",
                                         use_custom_kernels=False))
        captured: dict[str, list] = {}

        def hook(name):
            def fn(_mod, args, result):
                captured.setdefault(name, []).append((args[0].detach().clone(), result.detach().clone()))
            return fn

        for li, layer in enumerate(runner.model.model.layers):
            for p in PROJ:
                getattr(layer.self_attn, p).register_forward_hook(hook(f"l{li}.{p}"))
            layer.mlp.register_forward_hook(hook(f"l{li}.mlp"))

        prompt = [3, 17, 42, 5, 9, 61, 28, 11]
        seq = Sequence(seq_id=1, prompt_tokens=prompt,
                       sampling_params=SamplingParams(temperature=0.0, max_tokens=4),
                       metrics=RequestMetrics(enqueue_time=0.0))
        seq.prefill_progress = len(prompt)
        seq.status = "DECODING"
        plan = BatchPlan([BatchEntry(seq.seq_id, len(prompt), is_prefill_chunk=True)])
        logits_hook = {}
        runner.model.lm_head.register_forward_hook(
            lambda _m, _a, r: logits_hook.__setitem__("logits", r.detach().clone()))
        [(seq_id, token, _finished)] = runner.forward(plan, {seq.seq_id: seq})
        assert seq_id == 1

    for name, calls in captured.items():
        x, y = calls[0]
        out[f"{name}.x"] = x.reshape(-1, x.shape[-1]).numpy().astype(np.float32)
        out[f"{name}.y"] = y.reshape(-1, y.shape[-1]).numpy().astype(np.float32)
    out["prompt"] = np.array(prompt, dtype=np.int64)
    out["greedy_token"] = np.array([token], dtype=np.int64)
    out["last_logits"] = logits_hook["logits"][0, -1].numpy().astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "ref_tiny_llama_int8.npz"), **out)

    # Sanity: the oracle reproduces what the reference computed.
    for li in range(2):
        for p in PROJ:
            ref = ref_int8_linear(out[f"l{li}.{p}.x"], out[f"l{li}.{p}.q"], out[f"l{li}.{p}.s"])
            err = np.max(np.abs(ref - out[f"l{li}.{p}.y"])) / max(np.max(np.abs(ref)), 1e-30)
            assert err < 1e-5, (li, p, err)
    print("ref_tiny_llama_int8.npz: greedy token", token)


def config1_fixture() -> None:
    x, w, s = make_inputs(8, 2048, 2048, seed=0)
    y_oracle = ref_int8_linear(x.float().numpy(), w.numpy(), s.numpy())
    w_deq = (w.float() * s[:, None])
    y_ref_cpu = torch.nn.functional.linear(x.float(), w_deq).numpy()
    np.savez_compressed(
        os.path.join(HERE, "config1.npz"),
        sha_x=np.array(sha256(x)), sha_w=np.array(sha256(w)), sha_s=np.array(sha256(s)),
        y_oracle=y_oracle.astype(np.float32), y_ref_cpu=y_ref_cpu.astype(np.float32),
        x_head=x[:2, :16].float().numpy(), w_head=w[:2, :16].numpy(), s_head=s[:4].numpy(),
    )
    print("config1.npz written")


if __name__ == "__main__":
    ref_root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("LSE_REFERENCE_ROOT", "")
    if not ref_root or not os.path.isdir(ref_root):
        sys.exit("usage: make_golden.py <reference checkout>")
    config1_fixture()
    tiny_llama_fixture(ref_root)
