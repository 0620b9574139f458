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


def test_residual_binding_matches_the_reference_loop(tiny_dir, monkeypatch):
    """`bind_residual_epilogues` runs the reference's layer loop with each residual handed to the
    o_proj (through `attention_output`) and the MLP.  On the CPU, with stand-ins for the int8
    modules whose epilogue computes `residual + module(x)` in the reference's order, the hidden
    state is bit for bit the reference's `decoder_hidden`, and every layer hands both residuals
    over; an `attend` that calls o_proj itself (as `contiguous_attention` does) gets the
    reference's add; the piecewise runner's direct `attention_output` calls defer."""
    import torch

    runner = ModelRunner(ModelConfig(model_name_or_path=tiny_dir, device="cpu", dtype="float32",
                                     use_custom_kernels=False))
    calls = []

    class FakeLinear(torch.nn.Module):
        def __init__(self, inner):
            super().__init__()
            self.inner, self.out_features = inner, inner.out_features

        def forward(self, x, residual=None):
            calls.append(("o_proj", residual is not None))
            return self.inner(x) if residual is None else residual + self.inner(x)

    class FakeMLP(torch.nn.Module):
        def __init__(self, inner):
            super().__init__()
            self.inner = inner

        def forward(self, x, residual=None):
            calls.append(("mlp", residual is not None))
            return self.inner(x) if residual is None else residual + self.inner(x)

    monkeypatch.setattr(engine_hook, "Int8Linear", FakeLinear)
    monkeypatch.setattr(engine_hook, "Int8LlamaMLP", FakeMLP)
    g = torch.Generator().manual_seed(0)
    ids = torch.randint(1, 120, (1, 6), generator=g)
    pos = torch.arange(6).unsqueeze(0)
    nh, hd = runner.n_heads, runner.head_dim

    def heads(normed):  # any (1, T, H) -> (heads, T, head_dim) stand-in for attention
        return normed[0].view(normed.shape[1], nh, hd).transpose(0, 1)

    def via_output(normed, pe, i):
        return runner.attention_output(heads(normed), i)

    def direct(normed, pe, i):
        return runner._layers[i].self_attn.o_proj(heads(normed).transpose(0, 1).reshape(1, -1, nh * hd))

    with torch.no_grad():
        ref_a = runner.decoder_hidden(ids, pos, via_output)
        ref_b = runner.decoder_hidden(ids, pos, direct)
        for layer in runner._layers:
            layer.self_attn.o_proj = FakeLinear(layer.self_attn.o_proj)
            layer.mlp = FakeMLP(layer.mlp)
        engine_hook.bind_residual_epilogues(runner)
        engine_hook.bind_residual_epilogues(runner)  # idempotent
        calls.clear()
        assert torch.equal(runner.decoder_hidden(ids, pos, via_output), ref_a)
        n = len(runner._layers)
        assert calls == [("o_proj", True), ("mlp", True)] * n
        calls.clear()
        assert torch.equal(runner.decoder_hidden(ids, pos, direct), ref_b)
        assert calls == [("o_proj", False), ("mlp", True)] * n
        assert runner._lse_residual is None
        calls.clear()
        runner.attention_output(heads(torch.randn(1, 6, nh * hd, generator=g)), 0)
        assert calls == [("o_proj", False)]
