"""Drop-in modules on the GPU: the int8 projections of the reference's tiny Llama fixture
against the oracle, the fused QKV facades and MLP, a whole HF Llama quantized in place, and
CUDA-graph capture / replay (the reference captures decode and piecewise graphs around these
calls: decode_graph.py:87-116, piecewise_graph.py:71-109)."""

from __future__ import annotations

import os

import numpy as np
import pytest
import torch

from llm_serving_engine_b200.int8_linear import FusedInt8QKV, Int8Linear, Int8LlamaMLP, quantize_llama_
from oracle.ref_linear import ref_int8_linear, ref_mlp
from tests.gpu_helpers import check_parity

pytestmark = pytest.mark.gpu

PROJ = ("q_proj", "k_proj", "v_proj", "o_proj")


@pytest.fixture(scope="module")
def tiny(golden_dir):
    return dict(np.load(os.path.join(golden_dir, "ref_tiny_llama_int8.npz")))


def _bf16(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(a).to(torch.bfloat16)


@pytest.mark.parametrize("layer", [0, 1])
def test_reference_fixture_projections(tiny, layer):
    for p in PROJ:
        pre = f"l{layer}.{p}"
        x = _bf16(tiny[f"{pre}.x"])
        mod = Int8Linear.from_quantized(torch.from_numpy(tiny[f"{pre}.q"]).cuda(),
                                        torch.from_numpy(tiny[f"{pre}.s"]).cuda())
        y = mod(x.cuda())
        ref = ref_int8_linear(x.float().numpy(), tiny[f"{pre}.q"], tiny[f"{pre}.s"])
        check_parity(y, ref, pre)
        # and the reference's own fp32 nn.Linear output on the fp32 activations: the kernel
        # sees bf16-rounded x (relative error 2^-9 per element), so only the normwise bound
        # applies to this comparison
        yr = tiny[f"{pre}.y"].astype(np.float64)
        assert np.max(np.abs(y.float().cpu().numpy() - yr)) / np.max(np.abs(yr)) <= 1e-2, pre


@pytest.mark.parametrize("layer", [0, 1])
def test_reference_fixture_fused_qkv_and_mlp(tiny, layer):
    pre = f"l{layer}"
    qs = [torch.from_numpy(tiny[f"{pre}.{n}.q"]) for n in ("q_proj", "k_proj", "v_proj")]
    ss = [torch.from_numpy(tiny[f"{pre}.{n}.s"]) for n in ("q_proj", "k_proj", "v_proj")]
    fused = FusedInt8QKV(Int8Linear.from_quantized(torch.cat(qs).cuda(), torch.cat(ss).cuda()),
                         tuple(q.shape[0] for q in qs))
    qf, kf, vf = fused.facades()
    x = _bf16(tiny[f"{pre}.q_proj.x"]).cuda()
    outs = [qf(x), kf(x), vf(x)]
    for o, n in zip(outs, ("q_proj", "k_proj", "v_proj")):
        ref = ref_int8_linear(x.float().cpu().numpy(), tiny[f"{pre}.{n}.q"], tiny[f"{pre}.{n}.s"])
        check_parity(o, ref, f"{pre}.{n} fused")
    gate_up = Int8Linear.from_quantized(
        torch.cat([torch.from_numpy(tiny[f"{pre}.gate_proj.q"]), torch.from_numpy(tiny[f"{pre}.up_proj.q"])]).cuda(),
        torch.cat([torch.from_numpy(tiny[f"{pre}.gate_proj.s"]), torch.from_numpy(tiny[f"{pre}.up_proj.s"])]).cuda())
    down = Int8Linear.from_quantized(torch.from_numpy(tiny[f"{pre}.down_proj.q"]).cuda(),
                                     torch.from_numpy(tiny[f"{pre}.down_proj.s"]).cuda())
    mlp = Int8LlamaMLP(gate_up, down, tiny[f"{pre}.gate_proj.q"].shape[0])
    xm = _bf16(tiny[f"{pre}.mlp.x"])
    ref = ref_mlp(xm.float().numpy(), tiny[f"{pre}.gate_proj.q"], tiny[f"{pre}.gate_proj.s"],
                  tiny[f"{pre}.up_proj.q"], tiny[f"{pre}.up_proj.s"],
                  tiny[f"{pre}.down_proj.q"], tiny[f"{pre}.down_proj.s"])
    # bf16 rounding of the gate/up activations between the two projections adds ~1e-2
    y = mlp(xm.cuda()).float().cpu().numpy()
    assert np.max(np.abs(y - ref)) / np.max(np.abs(ref)) < 2e-2


def _tiny_llama(dtype=torch.bfloat16, hidden=256, inter=512, layers=2, heads=4, kv=2, vocab=128):
    from transformers import LlamaConfig, LlamaForCausalLM

    torch.manual_seed(0)
    cfg = LlamaConfig(vocab_size=vocab, hidden_size=hidden, intermediate_size=inter, num_hidden_layers=layers,
                      num_attention_heads=heads, num_key_value_heads=kv, max_position_embeddings=256,
                      bos_token_id=None, eos_token_id=None, pad_token_id=None)
    return LlamaForCausalLM(cfg).to(device="cuda", dtype=dtype).eval()


@torch.no_grad()
def test_quantized_hf_llama_matches_dequantized_float_model():
    model = _tiny_llama()
    quantize_llama_(model)
    # float twin with the dequantized weights
    twin = _tiny_llama(dtype=torch.float32)
    for lq, lf in zip(model.model.layers, twin.model.layers):
        qkv = lq.self_attn.qkv_int8
        w = qkv.fused.dequantized()
        sq, sk, _ = qkv.sizes
        lf.self_attn.q_proj.weight.copy_(w[:sq])
        lf.self_attn.k_proj.weight.copy_(w[sq:sq + sk])
        lf.self_attn.v_proj.weight.copy_(w[sq + sk:])
        lf.self_attn.o_proj.weight.copy_(lq.self_attn.o_proj.dequantized())
        lf.mlp.gate_proj.weight.copy_(lq.mlp.gate_weight())
        lf.mlp.up_proj.weight.copy_(lq.mlp.up_weight())
        lf.mlp.down_proj.weight.copy_(lq.mlp.down_proj.dequantized())
    twin.model.embed_tokens.weight.copy_(model.model.embed_tokens.weight.float())
    twin.lm_head.weight.copy_(model.lm_head.weight.float())
    for a, b in zip(model.model.layers, twin.model.layers):
        b.input_layernorm.weight.copy_(a.input_layernorm.weight.float())
        b.post_attention_layernorm.weight.copy_(a.post_attention_layernorm.weight.float())
    twin.model.norm.weight.copy_(model.model.norm.weight.float())
    ids = torch.randint(0, 128, (1, 24), device="cuda", generator=torch.Generator("cuda").manual_seed(1))
    lq = model(ids).logits.float()
    lf = twin(ids).logits
    err = (lq - lf).abs().max() / lf.abs().max()
    assert err < 3e-2, float(err)


@torch.no_grad()
def test_cuda_graph_capture_replays_int8_layers_exactly():
    """A decoder stack of int8 projections captured in one CUDA graph replays bit-identical
    to eager, for decode-sized (M=8) and prefill-sized (M=160) activations."""
    model = _tiny_llama(hidden=512, inter=1024, heads=8, kv=4)
    quantize_llama_(model)
    layers = model.model.layers
    pos_ids_cache = {}

    def step(h):
        for layer in layers:
            attn = layer.self_attn
            x = layer.input_layernorm(h)
            q, k, v = attn.q_proj(x), attn.k_proj(x), attn.v_proj(x)
            h = h + attn.o_proj(q + torch.cat([k, v], dim=-1).repeat(1, 1, 2)[..., : q.shape[-1]])
            h = h + layer.mlp(layer.post_attention_layernorm(h))
        return h

    for M in (8, 160):
        static_in = torch.randn(1, M, 512, device="cuda", dtype=torch.bfloat16)
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(3):  # warm-up on the capture stream, as the reference does
                step(static_in)
        torch.cuda.current_stream().wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            static_out = step(static_in)
        for trial in range(3):
            static_in.copy_(torch.randn(1, M, 512, device="cuda", dtype=torch.bfloat16))
            graph.replay()
            eager = step(static_in)
            torch.cuda.synchronize()
            assert torch.equal(static_out, eager), (M, trial)
        pos_ids_cache[M] = True


@torch.no_grad()
@pytest.mark.parametrize("fuse", [True, False])
def test_int8_checkpoint_save_load_reproduces_the_quantized_model(tmp_path, fuse):
    """quantize -> save -> load into a fresh model with the same non-projection weights:
    identical int8 weights and scales, and bit-identical logits."""
    from llm_serving_engine_b200.checkpoint import int8_state_dict, load_int8_checkpoint_, save_int8_checkpoint

    model = _tiny_llama()
    quantize_llama_(model, fuse=fuse)
    path = str(tmp_path / "int8.safetensors")
    save_int8_checkpoint(model, path)
    fresh = _tiny_llama()  # same seed: same embedding, norms and lm_head; float projections ignored
    load_int8_checkpoint_(fresh, path, fuse=fuse)
    a, _ = int8_state_dict(model)
    b, _ = int8_state_dict(fresh)
    for k in a:
        assert torch.equal(a[k], b[k]), k
    ids = torch.randint(0, 128, (1, 20), device="cuda", generator=torch.Generator("cuda").manual_seed(3))
    assert torch.equal(model(ids).logits, fresh(ids).logits)


@torch.no_grad()
def test_int8_lm_head_and_its_checkpoint(tmp_path):
    from llm_serving_engine_b200.checkpoint import load_int8_checkpoint_, save_int8_checkpoint

    model = _tiny_llama()
    head_w = model.lm_head.weight.detach().clone()
    quantize_llama_(model, lm_head=True)
    assert isinstance(model.lm_head, Int8Linear)
    err = (model.lm_head.dequantized() - head_w.float()).abs().max() / head_w.float().abs().max()
    assert err < 1e-2
    path = str(tmp_path / "int8_head.safetensors")
    save_int8_checkpoint(model, path)
    fresh = _tiny_llama()
    load_int8_checkpoint_(fresh, path)
    assert isinstance(fresh.lm_head, Int8Linear)
    ids = torch.randint(0, 128, (1, 12), device="cuda", generator=torch.Generator("cuda").manual_seed(4))
    assert torch.equal(model(ids).logits, fresh(ids).logits)
