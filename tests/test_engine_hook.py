"""Host-side behaviour of the `quantize="int8"` switch on the reference's ModelRunner (CPU).

The reference refuses int8 with NotImplementedError (`src/llm_serving_engine/model/
model_runner.py:45-46`, pinned by its `tests/test_model_runner.py:120-122`).  With
`engine_hook.install()` the same call loads an int8 model on a GPU (tests/test_gpu_engine.py);
on a machine without CUDA it must refuse loudly instead of falling back to a CPU path, and
every other config must run the reference's own constructor unchanged.
"""

from __future__ import annotations

import pytest

from tests.engine_helpers import ModelConfig, ModelRunner, save_tiny_llama

from llm_serving_engine_b200 import engine_hook


@pytest.fixture(scope="module")
def tiny_dir(tmp_path_factory):
    return save_tiny_llama(tmp_path_factory.mktemp("tiny-int8-llama-cpu"))


@pytest.fixture
def hooked():
    engine_hook.install()
    yield
    engine_hook.uninstall()


def test_reference_refuses_int8_without_the_hook(tiny_dir):
    assert not engine_hook.installed()
    with pytest.raises(NotImplementedError):
        ModelRunner(ModelConfig(model_name_or_path=tiny_dir, device="cpu", quantize="int8", use_custom_kernels=False))


def test_hook_refuses_int8_without_cuda(tiny_dir, hooked, monkeypatch):
    import torch

    monkeypatch.setattr(torch.cuda, "is_available", lambda: False)
    with pytest.raises(RuntimeError, match="needs a CUDA device"):
        ModelRunner(ModelConfig(model_name_or_path=tiny_dir, device="cuda", quantize="int8"))


def test_hook_leaves_other_configs_to_the_reference(tiny_dir, hooked):
    runner = ModelRunner(ModelConfig(model_name_or_path=tiny_dir, device="cpu", dtype="float32",
                                     use_custom_kernels=False))
    assert runner.config.quantize == "none"
    assert type(runner.model.model.layers[0].self_attn.o_proj).__name__ == "Linear"


def test_install_is_idempotent_and_uninstall_restores():
    original = ModelRunner.__init__
    engine_hook.install()
    wrapped = ModelRunner.__init__
    engine_hook.install()
    assert ModelRunner.__init__ is wrapped and wrapped is not original
    engine_hook.uninstall()
    assert ModelRunner.__init__ is original
    assert not engine_hook.installed()


def test_rope_binding_defers_to_the_reference_without_a_fused_int8_qkv(tiny_dir):
    """`bind_rope_kv_write` only takes layers that carry a fused int8 QKV (in bf16); any other
    layer runs the reference's own `write_kv_and_project_q`, with the same arguments."""
    import torch

    runner = ModelRunner(ModelConfig(model_name_or_path=tiny_dir, device="cpu", dtype="float32",
                                     use_custom_kernels=False))
    calls = []
    runner.write_kv_and_project_q = lambda *args: calls.append(args) or "reference"
    engine_hook.bind_rope_kv_write(runner)
    normed = torch.zeros(1, 3, 256)
    out = runner.write_kv_and_project_q(normed, (None, None), 0, "blocks", "within")
    assert out == "reference" and len(calls) == 1
    assert calls[0][0] is normed and calls[0][2:] == (0, "blocks", "within")


def test_norm_binding_wraps_every_norm_once_and_defers_on_cpu(tiny_dir):
    """`bind_rms_norms` puts the kernel-served module in every RMSNorm slot (idempotently);
    rows it cannot serve (here fp32 on the CPU) go to the module it replaced, unchanged."""
    import torch

    runner = ModelRunner(ModelConfig(model_name_or_path=tiny_dir, device="cpu", dtype="float32",
                                     use_custom_kernels=False))
    layer = runner.model.model.layers[0]
    x = torch.randn(1, 3, 256)
    before = layer.input_layernorm(x)
    engine_hook.bind_rms_norms(runner)
    engine_hook.bind_rms_norms(runner)
    assert type(layer.input_layernorm).__name__ == "_KernelRMSNorm"
    assert type(layer.input_layernorm.original).__name__ == "LlamaRMSNorm"
    assert type(runner.model.model.norm).__name__ == "_KernelRMSNorm"
    assert all(type(lay.post_attention_layernorm).__name__ == "_KernelRMSNorm" for lay in runner.model.model.layers)
    assert torch.equal(layer.input_layernorm(x), before)
