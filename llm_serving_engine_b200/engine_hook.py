"""The reference engine's `quantize="int8"` switch, bound to this package.

The reference selects int8 with `ModelConfig.quantize = "int8"` (`LLM_QUANTIZE=int8`,
`src/llm_serving_engine/config.py:32,46`) and refuses it as the first statement of
`ModelRunner.__init__` (`src/llm_serving_engine/model/model_runner.py:45-46`).  A maintainer
binds the switch by replacing that raise with the post-load swap `enable_int8(self)` (the
two-line hook shown in the integration notes).  `install()` does the same from outside, for
a reference that has not been edited: it wraps `ModelRunner.__init__` so that a config with
`quantize="int8"` loads the model as the reference does (with `quantize="none"`), then swaps
the projections, and any other config runs the reference's `__init__` untouched.

After the swap nothing else in the engine changes: `forward`, `forward_fused`,
`DecodeGraphRunner` (`decode_graph.py:87-140`) and `PiecewiseGraphRunner`
(`piecewise_graph.py:71-183`) call the same module slots.  The runner's paged attention
(`ModelRunner.attend_paged`, `model_runner.py:357-363`, reached from `paged_attention` in the
eager and decode-graph paths and from the piecewise runner between its segments) is bound to
this package's kernel on the same arguments (`ops.paged_attention`, the drop-in for the
reference's Triton `paged_attention_forward`).  `decoder_hidden` and `attention_output`
(eager and decode-graph paths) are bound to forms that add each layer's residual in the int8
o_proj and down epilogues (same layer order; the sum is rounded once instead of twice).
int8 needs CUDA; on a CPU-only
machine the switch raises `RuntimeError` at load, the way the reference's custom-kernel
check refuses a CPU device (`model_runner.py:77-94`); there is no CPU fallback.
"""

from __future__ import annotations

import dataclasses
import functools

import torch

from . import ops
from .int8_linear import Int8Linear, Int8LlamaMLP, quantize_llama_

__all__ = ["enable_int8", "bind_paged_attention", "bind_rope_kv_write", "bind_rms_norms", "bind_residual_epilogues",
           "install", "uninstall", "installed"]


def _attend_paged(runner, q, layer_idx, paging):
    """`ModelRunner.attend_paged` on this package's kernels: same arguments, same result.  A
    batch of single-token entries (every decode step; their rows are the entries in order) in
    bf16 or fp16 takes the decode kernel, unsplit (no workspace, so any capture stream records it); any
    other batch the multi-token kernel."""
    k_pool, v_pool = runner._k_pool[layer_idx], runner._v_pool[layer_idx]
    E = paging.block_table.shape[0]
    if paging.max_q_len == 1 and q.shape[1] == E and q.dtype in (torch.bfloat16, torch.float16):
        max_context = paging.block_table.shape[1] * runner._block_size
        o = ops.paged_decode_attention(q.transpose(0, 1), k_pool, v_pool, paging.block_table, paging.context_len,
                                       max_context, split=False)
        return o.transpose(0, 1)
    return ops.paged_attention(q, k_pool, v_pool, paging.block_table, paging.context_len, paging.query_offset,
                               paging.q_start, paging.q_len, runner._block_size, paging.max_q_len)


def _write_kv_and_project_q(runner, original, normed, position_embeddings, layer_idx, dest_block_id, dest_within):
    """`ModelRunner.write_kv_and_project_q` (`model_runner.py:342-355`) as two launches: the
    layer's fused int8 QKV projection, then one kernel that rotates q and k (rotate-half RoPE
    in fp32, one rounding), writes k and v into their pool slots and returns q as (heads,
    tokens, head_dim).  Layers without a fused int8 QKV, and dtypes other than bf16 and fp16,
    take the reference's own code."""
    attn = runner._layers[layer_idx].self_attn
    qkv_mod = getattr(attn, "qkv_int8", None)
    if qkv_mod is None or normed.dtype not in (torch.bfloat16, torch.float16):
        return original(normed, position_embeddings, layer_idx, dest_block_id, dest_within)
    cos, sin = position_embeddings
    T = normed.shape[1]
    qkv = qkv_mod.fused(normed[0])  # [T, (H + 2 H_kv) * D]
    k_pool, v_pool = runner._k_pool[layer_idx], runner._v_pool[layer_idx]
    off = ops.pool_slot_offsets(dest_block_id, dest_within, k_pool)
    return ops.rope_kv_write(qkv, runner.n_heads, runner.n_kv_heads, runner.head_dim, cos[0].reshape(T, -1),
                             sin[0].reshape(T, -1), k_pool, v_pool, off)


def bind_rope_kv_write(runner):
    """Route the runner's `write_kv_and_project_q` (the K/V write and q of paged attention, in
    the eager, decode-graph and piecewise paths) through the fused QKV projection and this
    package's RoPE + K/V write kernel (an instance attribute, as `bind_paged_attention`)."""
    runner.write_kv_and_project_q = functools.partial(_write_kv_and_project_q, runner,
                                                      runner.write_kv_and_project_q)
    return runner


class _KernelRMSNorm(torch.nn.Module):
    """A LlamaRMSNorm slot served by the one-launch RMSNorm kernel (`ops.rms_norm`: the same
    roundings as transformers' module, the fp32 mean in another order) for bf16 and fp16 CUDA
    rows;
    any other input goes to the module it replaced."""

    def __init__(self, original: torch.nn.Module):
        super().__init__()
        self.original = original
        self.weight = original.weight
        self.eps = float(getattr(original, "variance_epsilon", getattr(original, "eps", 1e-6)))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.is_cuda and x.dtype in (torch.bfloat16, torch.float16) and self.weight.dtype == x.dtype:
            return ops.rms_norm(x, self.weight, self.eps)
        return self.original(x)


def bind_rms_norms(runner):
    """Serve every decoder layer's `input_layernorm` / `post_attention_layernorm` and the final
    norm (`model_runner.py:213-224`) with the RMSNorm kernel: one launch each instead of
    torch's seven.  Idempotent."""
    def wrap(module):
        return module if isinstance(module, _KernelRMSNorm) else _KernelRMSNorm(module)

    for layer in runner._layers:
        layer.input_layernorm = wrap(layer.input_layernorm)
        layer.post_attention_layernorm = wrap(layer.post_attention_layernorm)
    runner.model.model.norm = wrap(runner.model.model.norm)
    return runner


def _attention_output(runner, original, attn, layer_idx):
    """`ModelRunner.attention_output` (`model_runner.py:365-369`) with the layer's residual added
    in the int8 o_proj's epilogue when the bound `decoder_hidden` left it for this layer;
    otherwise (the piecewise runner between its segments, a float o_proj, a foreign shape) the
    reference's own code."""
    pending = runner._lse_residual
    o_proj = runner._layers[layer_idx].self_attn.o_proj
    T = attn.shape[1]
    if (pending is None or pending[0] != layer_idx or not isinstance(o_proj, Int8Linear)
            or pending[1].shape != (1, T, o_proj.out_features) or pending[1].dtype != attn.dtype):
        return original(attn, layer_idx)
    runner._lse_residual = None
    out = attn.transpose(0, 1).reshape(1, T, runner.n_heads * runner.head_dim)
    return o_proj(out, residual=pending[1])


def _decoder_hidden(runner, original, input_ids, position_ids, attend):
    """`ModelRunner.decoder_hidden` (`model_runner.py:213-224`) with each layer's two residual
    adds in the epilogues of its int8 projections: `hidden + o_proj(attn)` and
    `hidden + mlp(normed)` each come out of the projection kernel rounded once, instead of a
    projection output plus an elementwise add (two launches fewer per layer).  o_proj runs
    inside `attend` (`attention_output`), so the residual is left for it there; when `attend`
    does not take it (`contiguous_attention` calls o_proj itself) or a slot is not int8, the add
    runs as the reference writes it."""
    model = runner.model
    hidden = model.get_input_embeddings()(input_ids)
    position_embeddings = model.model.rotary_emb(hidden, position_ids)
    for layer_idx, layer in enumerate(runner._layers):
        runner._lse_residual = (layer_idx, hidden)
        try:
            out = attend(layer.input_layernorm(hidden), position_embeddings, layer_idx)
            taken = runner._lse_residual is None
        finally:
            runner._lse_residual = None
        hidden = out if taken else hidden + out
        normed = layer.post_attention_layernorm(hidden)
        hidden = layer.mlp(normed, residual=hidden) if isinstance(layer.mlp, Int8LlamaMLP) else hidden + layer.mlp(normed)
    return model.model.norm(hidden)


def bind_residual_epilogues(runner):
    """Route the runner's `decoder_hidden` (the eager and decode-graph paths) and
    `attention_output` through the fused residual epilogues (instance attributes, as
    `bind_paged_attention`).  Idempotent."""
    if getattr(runner, "_lse_residual_bound", False):
        return runner
    runner._lse_residual = None
    runner.attention_output = functools.partial(_attention_output, runner, runner.attention_output)
    runner.decoder_hidden = functools.partial(_decoder_hidden, runner, runner.decoder_hidden)
    runner._lse_residual_bound = True
    return runner


def bind_paged_attention(runner):
    """Route the runner's paged attention to `ops.paged_attention` (an instance attribute, so
    the runner's own `paged_attention` and the graph runners call it)."""
    runner.attend_paged = functools.partial(_attend_paged, runner)
    return runner


def enable_int8(runner, lm_head: bool = False, attention: bool = True, rope: bool = True, norms: bool = True,
                residuals: bool = True):
    """Swap a loaded `ModelRunner`'s projections to int8 in place.  `runner.model` is the
    Llama-family model the runner loaded; every decoder layer's q/k/v (one fused int8 QKV),
    o_proj and MLP become int8 (`quantize_llama_`), and the lm_head too with `lm_head=True`;
    with `attention=True` the paged attention runs on this package's kernel too, and with
    `rope=True` the K/V write and q (`write_kv_and_project_q`) on the fused QKV projection and
    the RoPE + K/V write kernel, with `norms=True` the RMSNorms on the RMSNorm kernel, and with
    `residuals=True` the decoder's residual adds in the o_proj and down epilogues.
    Nothing else needs preparing: the ops hold no per-stream
    state, so the engine's graph captures on any stream record them as they are."""
    device = torch.device(runner.device)
    if device.type != "cuda":
        raise RuntimeError(f"int8 weight-only quantization needs a CUDA device, got {runner.device!r}")
    quantize_llama_(runner.model, lm_head=lm_head)
    if attention:
        bind_paged_attention(runner)
    if rope:
        bind_rope_kv_write(runner)
    if norms:
        bind_rms_norms(runner)
    if residuals:
        bind_residual_epilogues(runner)
    return runner


def _check_cuda(config) -> None:
    if not torch.cuda.is_available() or not str(config.device).startswith("cuda"):
        raise RuntimeError(
            f"int8 weight-only quantization needs a CUDA device (config.device={config.device!r}, "
            f"cuda available: {torch.cuda.is_available()}); there is no CPU int8 path")


def _runner_class():
    from llm_serving_engine.model.model_runner import ModelRunner

    return ModelRunner


def installed() -> bool:
    return getattr(_runner_class().__init__, "_lse_int8", False)


def install(lm_head: bool = False, rope: bool = True, norms: bool = True, residuals: bool = True) -> None:
    """Make `ModelRunner(ModelConfig(quantize="int8"))` load an int8 model (idempotent; the
    options of the first call stay until `uninstall`)."""
    cls = _runner_class()
    if installed():
        return
    original = cls.__init__

    @functools.wraps(original)
    def __init__(self, config, *args, **kwargs):
        if getattr(config, "quantize", "none") != "int8":
            return original(self, config, *args, **kwargs)
        _check_cuda(config)
        original(self, dataclasses.replace(config, quantize="none"), *args, **kwargs)
        self.config = config
        enable_int8(self, lm_head=lm_head, rope=rope, norms=norms, residuals=residuals)

    __init__._lse_int8 = True
    __init__._lse_original = original
    cls.__init__ = __init__


def uninstall() -> None:
    """Restore the reference's own `ModelRunner.__init__`."""
    cls = _runner_class()
    if installed():
        cls.__init__ = cls.__init__._lse_original
