"""Drop-in int8 modules for the reference engine's projections.

The reference reaches its projections as modules in fixed attribute slots and calls them
with one activation `(1, M, hidden)`:

* `layer.self_attn.q_proj/k_proj/v_proj(normed)` in `ModelRunner._project_qkv`
  (`src/llm_serving_engine/model/model_runner.py:322-324`), and in HF's own
  `LlamaAttention.forward`;
* `layer.self_attn.o_proj(out)` in `attention_output` / `contiguous_attention`
  (`model_runner.py:369`, `:418`);
* `layer.mlp(x)` in `decoder_hidden` (`model_runner.py:223`) and in the piecewise graph
  segments (`src/llm_serving_engine/model/piecewise_graph.py:163-166`).

`quantize_llama_(model)` swaps those slots in place:

* `Int8Linear` replaces one `nn.Linear` (same `__call__(x[..., K]) -> [..., N]` contract);
* `FusedInt8QKV` holds ONE int8 weight `[q; k; v]` (N = (H + 2*Hkv) * hd) and installs three
  small facades in the `q_proj/k_proj/v_proj` slots: calling `q_proj(x)` runs the fused
  projection once and `k_proj(x)` / `v_proj(x)` on the same `x` return column views of it,
  so callers that invoke the three projections in sequence (the runner, HF attention) run one
  kernel and stay unchanged;
* `Int8LlamaMLP` replaces `layer.mlp`: one fused gate_up int8 projection (N = 2 * I, gate and
  up rows interleaved in 8-row blocks), SiLU*mul (in the decode kernel's epilogue for up to
  16 tokens), and the int8 down projection - transformers' `LlamaMLP.forward`
  (`down(act(gate(x)) * up(x))`).

Weights are quantized on the GPU at load (`ops.quantize_per_channel`), once.  Activations
are bf16 in and out; a fp16/fp32 model's activations are cast to bf16 for the kernel and the
result cast back, so the modules drop into any model dtype.
"""

from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import ops

__all__ = ["Int8Linear", "FusedInt8QKV", "Int8LlamaMLP", "quantize_llama_", "int8_weight_bytes"]


_NATIVE = (torch.bfloat16, torch.float16)


def _to_bf16(x: torch.Tensor) -> torch.Tensor:
    return x if x.dtype == torch.bfloat16 else x.to(torch.bfloat16)


class Int8Linear(nn.Module):
    """`y = x @ (W * scale[:, None]).T` with int8 `W [N, K]`, fp32 `scale [N]`.

    W is kept only in the tile-contiguous packed layout the kernels stream
    (`ops.pack_weight`: every 128 x 128 tile is 16 KB of contiguous memory); `weight`
    unpacks it on demand for inspection.
    """

    def __init__(self, in_features: int, out_features: int, device=None):
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        nbytes = ops.packed_weight_bytes(out_features, in_features) if device is not None and torch.device(device).type == "cuda" else 0
        self.register_buffer("weight_packed", torch.zeros((nbytes,), dtype=torch.int8, device=device))
        self.register_buffer("scale", torch.ones((out_features,), dtype=torch.float32, device=device))

    @classmethod
    def from_quantized(cls, weight: torch.Tensor, scale: torch.Tensor) -> "Int8Linear":
        """From an int8 [N, K] weight and fp32 [N] scale already on the GPU."""
        mod = cls(weight.shape[1], weight.shape[0], device=None)
        mod.weight_packed = ops.pack_weight(weight)
        mod.scale = scale.to(torch.float32).contiguous()
        return mod

    @classmethod
    def from_linear(cls, linear: nn.Linear) -> "Int8Linear":
        if linear.bias is not None:
            raise ValueError("Int8Linear: biased projections are not supported (Llama has none)")
        q, s = ops.quantize_per_channel(linear.weight.detach())
        return cls.from_quantized(q, s)

    @classmethod
    def from_float_weights(cls, *weights: torch.Tensor) -> "Int8Linear":
        """Quantize the row-concatenation of `weights` (fused projections)."""
        w = torch.cat([t.detach() for t in weights], dim=0) if len(weights) > 1 else weights[0].detach()
        q, s = ops.quantize_per_channel(w)
        return cls.from_quantized(q, s)

    @property
    def weight(self) -> torch.Tensor:
        return ops.unpack_weight(self.weight_packed, self.out_features, self.in_features)

    def dequantized(self, dtype: torch.dtype = torch.float32) -> torch.Tensor:
        return (self.weight.to(torch.float32) * self.scale[:, None]).to(dtype)

    def forward(self, x: torch.Tensor, residual: torch.Tensor | None = None) -> torch.Tensor:
        """`x @ W.T`, or `residual + x @ W.T` rounded once (the decoder's residual add fused
        into the kernel).  bf16 and fp16 activations run natively (one `lse::int8_linear`
        dispatcher call); other dtypes go through bf16."""
        if x.dtype in _NATIVE and (residual is None or residual.dtype == x.dtype):
            return ops.torch_ops().int8_linear(x, self.weight_packed, self.scale, self.out_features, self.in_features,
                                               residual)
        if residual is not None:
            return residual + self.forward(x)
        return self.forward(_to_bf16(x)).to(x.dtype)

    def extra_repr(self) -> str:
        return f"in_features={self.in_features}, out_features={self.out_features}, int8 per-channel, packed"


class _SliceOf(nn.Module):
    """Facade in a q_proj/k_proj/v_proj slot: a column range of the fused QKV output."""

    def __init__(self, parent: "FusedInt8QKV", index: int):
        super().__init__()
        self._parent = [parent]  # not a submodule: avoids a reference cycle in the module tree
        self.index = index
        self.in_features = parent.fused.in_features
        self.out_features = parent.sizes[index]

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self._parent[0].part(x, self.index)


class FusedInt8QKV(nn.Module):
    """One int8 projection for q, k and v (N = q + k + v columns)."""

    def __init__(self, fused: Int8Linear, sizes: tuple[int, int, int]):
        super().__init__()
        assert sum(sizes) == fused.out_features
        self.fused = fused
        self.sizes = tuple(sizes)
        self._last_key = None
        self._last_out: list[torch.Tensor] | None = None

    @classmethod
    def from_linears(cls, q: nn.Linear, k: nn.Linear, v: nn.Linear) -> "FusedInt8QKV":
        for lin in (q, k, v):
            if lin.bias is not None:
                raise ValueError("FusedInt8QKV: biased projections are not supported")
        fused = Int8Linear.from_float_weights(q.weight, k.weight, v.weight)
        return cls(fused, (q.out_features, k.out_features, v.out_features))

    def forward(self, x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        y = self.fused(x)
        return tuple(torch.split(y, self.sizes, dim=-1))

    def part(self, x: torch.Tensor, index: int) -> torch.Tensor:
        # The q projection (index 0) always recomputes; k and v reuse it when called on the
        # very same activation (same storage, shape and version), which is how both the
        # reference runner and HF attention call them.
        key = (x.data_ptr(), tuple(x.shape), x.stride(), x._version, x.device)
        if index == 0 or self._last_out is None or key != self._last_key:
            self._last_out = list(self.forward(x))
            self._last_key = key
        out = self._last_out[index]
        if index == 2:
            self._last_out, self._last_key = None, None
        return out

    def facades(self) -> tuple[_SliceOf, _SliceOf, _SliceOf]:
        return _SliceOf(self, 0), _SliceOf(self, 1), _SliceOf(self, 2)


class Int8LlamaMLP(nn.Module):
    """`down(silu(gate(x)) * up(x))` with a fused int8 gate_up and an int8 down projection.

    gate_up holds the gate and up rows interleaved in 8-row blocks (`ops.interleave_gate_up_rows`),
    so for up to 16 tokens one kernel computes both projections and SiLU * mul
    (`ops.int8_gate_up_silu_packed`); above that the tensor-core kernel computes the
    interleaved [M, 2I] projection and the columns are paired here.
    """

    def __init__(self, gate_up: Int8Linear, down: Int8Linear, intermediate: int, act=F.silu,
                 interleaved: bool = False):
        super().__init__()
        if not interleaved:  # [gate; up] rows -> 16-row blocks interleaved
            perm = ops.interleave_gate_up_rows(intermediate, device=gate_up.scale.device)
            gate_up = Int8Linear.from_quantized(gate_up.weight.index_select(0, perm), gate_up.scale.index_select(0, perm))
        self.gate_up = gate_up
        self.down_proj = down
        self.intermediate_size = intermediate
        self.act = act

    @classmethod
    def from_quantized(cls, q_gate_up: torch.Tensor, s_gate_up: torch.Tensor, q_down: torch.Tensor,
                       s_down: torch.Tensor, intermediate: int, act=F.silu) -> "Int8LlamaMLP":
        """From int8 weights already on the GPU: `q_gate_up [2I, H]` in [gate; up] row order
        with its scales, and `q_down [H, I]` with its scales."""
        perm = ops.interleave_gate_up_rows(intermediate, device=q_gate_up.device)
        gate_up = Int8Linear.from_quantized(q_gate_up.index_select(0, perm), s_gate_up.index_select(0, perm))
        return cls(gate_up, Int8Linear.from_quantized(q_down, s_down), intermediate, act, interleaved=True)

    @classmethod
    def from_mlp(cls, mlp: nn.Module) -> "Int8LlamaMLP":
        gate, up, down = mlp.gate_proj, mlp.up_proj, mlp.down_proj
        for lin in (gate, up, down):
            if lin.bias is not None:
                raise ValueError("Int8LlamaMLP: biased projections are not supported")
        act = getattr(mlp, "act_fn", F.silu)
        gate_up = Int8Linear.from_float_weights(gate.weight, up.weight)
        return cls(gate_up, Int8Linear.from_linear(down), gate.out_features, act)

    def split_rows(self, t: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """(gate rows, up rows) of a tensor [2I, ...] in the interleaved row order."""
        v = t.view(self.intermediate_size // 8, 2, 8, *t.shape[1:])
        return v[:, 0].reshape(self.intermediate_size, *t.shape[1:]), v[:, 1].reshape(self.intermediate_size, *t.shape[1:])

    def gate_weight(self, dtype: torch.dtype = torch.float32) -> torch.Tensor:
        """Dequantized gate_proj weight [I, H]."""
        return self.split_rows(self.gate_up.dequantized(dtype))[0]

    def up_weight(self, dtype: torch.dtype = torch.float32) -> torch.Tensor:
        """Dequantized up_proj weight [I, H]."""
        return self.split_rows(self.gate_up.dequantized(dtype))[1]

    def _silu(self) -> bool:
        # torch's SiLU, or transformers' SiLUActivation (ACT2FN["silu"], x * sigmoid(x))
        return self.act is F.silu or type(self.act).__name__ in ("SiLU", "SiLUActivation")

    def forward(self, x: torch.Tensor, residual: torch.Tensor | None = None) -> torch.Tensor:
        """`down(act(gate(x)) * up(x))`, plus `residual` added in the down projection's
        epilogue when given.  bf16 and fp16 run natively; other dtypes go through bf16."""
        if x.dtype not in _NATIVE or (residual is not None and residual.dtype != x.dtype):
            if residual is not None:
                return residual + self.forward(x)
            return self.forward(_to_bf16(x)).to(x.dtype)
        I = self.intermediate_size
        if self._silu():
            h = ops.torch_ops().gate_up_silu(x, self.gate_up.weight_packed, self.gate_up.scale, I,
                                             self.gate_up.in_features)
        else:
            gu = self.gate_up(x).view(*x.shape[:-1], I // 8, 2, 8)
            h = (self.act(gu[..., 0, :]) * gu[..., 1, :]).reshape(*x.shape[:-1], I)
        return self.down_proj(h, residual=residual)


def quantize_llama_(model: nn.Module, fuse: bool = True, lm_head: bool = False) -> nn.Module:
    """In place: every decoder layer's q/k/v/o and MLP projections become int8.

    `model` is a Llama-family `*ForCausalLM` on a CUDA device (the layout
    `ModelRunner.check_custom_kernel_support` requires, `model_runner.py:77-94`).  The
    embedding stays in the model dtype; so does the lm_head unless `lm_head=True`, which
    makes it an `Int8Linear` too (vocab x hidden, the largest single matrix of the decode
    step; it breaks a tie with the input embedding, which keeps its own weight).
    """
    decoder = getattr(model, "model", model)
    layers = getattr(decoder, "layers", None)
    if layers is None:
        raise RuntimeError(f"int8: {type(model).__name__} has no Llama-family decoder layers (model.model.layers)")
    for layer in layers:
        attn = layer.self_attn
        if fuse:
            qkv = FusedInt8QKV.from_linears(attn.q_proj, attn.k_proj, attn.v_proj)
            attn.qkv_int8 = qkv
            attn.q_proj, attn.k_proj, attn.v_proj = qkv.facades()
        else:
            attn.q_proj = Int8Linear.from_linear(attn.q_proj)
            attn.k_proj = Int8Linear.from_linear(attn.k_proj)
            attn.v_proj = Int8Linear.from_linear(attn.v_proj)
        attn.o_proj = Int8Linear.from_linear(attn.o_proj)
        layer.mlp = Int8LlamaMLP.from_mlp(layer.mlp)
    if lm_head:
        head = getattr(model, "lm_head", None)
        if not isinstance(head, nn.Linear):
            raise RuntimeError(f"int8: {type(model).__name__} has no nn.Linear lm_head")
        model.lm_head = Int8Linear.from_linear(head)
    torch.cuda.empty_cache()
    return model


def int8_weight_bytes(model: nn.Module) -> int:
    """Bytes of int8 weights + fp32 scales the quantized layers stream per forward."""
    total = 0
    for mod in model.modules():
        if isinstance(mod, Int8Linear):
            total += mod.out_features * mod.in_features + 4 * mod.scale.numel()
    return total
