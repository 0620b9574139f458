"""Batched decode step of a Llama-3-style decoder on the int8 projections: the vehicle for
the end-to-end decode measurement (decode tokens/s with int8 vs bf16 projection weights).

The step follows the reference's graphed decode step (src/llm_serving_engine/model/
decode_graph.py:125-140 over `decoder_hidden`, model_runner.py:213-224): embedding, then per
layer RMSNorm -> fused QKV -> RoPE -> K/V write -> attention over the sequence's cache ->
o_proj -> residual -> RMSNorm -> gate_up -> SiLU * mul -> down -> residual, then the final
norm, the lm_head and the greedy token.  The projections are this package's int8 modules
(`quantize=True`) or bf16 `F.linear` on the same random weights (`quantize=False`, the
reference's `quantize="none"`).

Attention (`attention="paged"`, the default) runs this package's sm_100a paged decode
kernel (`ops.paged_decode_attention`) over K/V pools in the reference's layout
([num_blocks, block_size, H_kv, head_dim] per layer, a shuffled block table, one spare
block); `attention="sdpa"` keeps one contiguous [B, H_kv, context + 1, head_dim] cache per
layer and torch's scaled_dot_product_attention, for comparison.

Stated differences from the reference engine (none of them on the int8 path):
  * a timed step keeps its position fixed: it writes the new K/V into slot `context` and
    attends over all context + 1 positions, so the CUDA graph's shapes are static and every
    replay does exactly the work of a decode step at that context length.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F

from . import ops
from .int8_linear import Int8Linear, Int8LlamaMLP

__all__ = ["LlamaShape", "LLAMA3_8B", "DecodeModel", "decode_bytes_per_step"]


@dataclass(frozen=True)
class LlamaShape:
    layers: int
    hidden: int
    heads: int
    kv_heads: int
    head_dim: int
    intermediate: int
    vocab: int
    rope_theta: float = 500000.0
    eps: float = 1e-5


LLAMA3_8B = LlamaShape(layers=32, hidden=4096, heads=32, kv_heads=8, head_dim=128, intermediate=14336, vocab=128256)


def decode_bytes_per_step(shape: LlamaShape, batch: int, context: int, quantize: bool,
                          int8_lm_head: bool = False) -> int:
    """HBM bytes one decode step must read at least: projection weights (int8 + fp32 scales,
    or bf16), the K/V of every sequence (context + 1 positions), the lm_head (bf16, or int8
    + scales) and the new tokens' embedding rows."""
    H, hd = shape.hidden, shape.head_dim
    n_qkv = (shape.heads + 2 * shape.kv_heads) * hd
    per_layer = [(H, n_qkv), (shape.heads * hd, H), (H, 2 * shape.intermediate), (shape.intermediate, H)]
    w = sum(k * n * (1 if quantize else 2) + (4 * n if quantize else 0) for k, n in per_layer) * shape.layers
    kv = 2 * shape.layers * batch * shape.kv_heads * (context + 1) * hd * 2
    head = shape.vocab * H + 4 * shape.vocab if int8_lm_head else shape.vocab * H * 2
    return w + kv + head + batch * H * 2


def _rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    return ops.rms_norm(x, w, eps)  # one sm_100a kernel instead of torch's seven


def _bf16_mlp(x: torch.Tensor, w_gate_up: torch.Tensor, w_down: torch.Tensor, inter: int) -> torch.Tensor:
    gu = F.linear(x, w_gate_up)
    return F.linear(F.silu(gu[:, :inter]) * gu[:, inter:], w_down)


class DecodeModel:
    """Random-init Llama decoder for `batch` sequences at `context` cached positions."""

    def __init__(self, shape: LlamaShape, batch: int, context: int, device, seed: int = 0,
                 quantize: bool = True, weights: list | None = None, quantize_lm_head: bool = False,
                 attention: str = "paged", kv: dict | None = None, block_size: int = 16, fuse_norms: bool = False):
        if attention not in ("paged", "sdpa"):
            raise ValueError(f"attention must be 'paged' or 'sdpa', got {attention!r}")
        self.shape, self.batch, self.context, self.quantize = shape, batch, context, quantize
        self.attention, self.block_size = attention, block_size
        # int8 with fuse_norms: each layer's two RMSNorms run fused into the projections that
        # consume them (ops.rms_norm_proj, one launch fewer each).  Off by default: measured on
        # B200 at 64 sequences, 5.20 ms/step fused against 5.17 ms separate -- the projection's
        # weight copies already stream under the norm and split kernels (programmatic dependent
        # launch), so removing one of them shortens nothing.
        self.fuse_norms = fuse_norms
        dev = torch.device(device)
        g = torch.Generator(device=dev).manual_seed(seed)

        def w(*size):
            return (torch.randn(*size, generator=g, device=dev) * 0.02).to(torch.bfloat16)

        H, hd, I = shape.hidden, shape.head_dim, shape.intermediate
        self.embed = w(shape.vocab, H)
        self.lm_head = w(shape.vocab, H)
        self.final_norm = torch.ones(H, device=dev, dtype=torch.bfloat16)
        # bf16 weights per layer: [q;k;v], o, [gate;up], down (shared with a quantized twin)
        self.weights = weights if weights is not None else [
            (torch.cat([w(shape.heads * hd, H), w(2 * shape.kv_heads * hd, H)]), w(H, shape.heads * hd),
             torch.cat([w(I, H), w(I, H)]), w(H, I)) for _ in range(shape.layers)]
        # per layer: (qkv, o, mlp) callables, o and mlp taking the residual stream; the int8
        # modules add it in their kernels' epilogue, and the int8 MLP stores gate/up
        # interleaved and runs the fused gate_up + SiLU * mul kernel for up to 16 sequences
        if quantize:
            self.proj = [(Int8Linear.from_float_weights(wqkv), Int8Linear.from_float_weights(wo),
                          Int8LlamaMLP(Int8Linear.from_float_weights(wgu), Int8Linear.from_float_weights(wd), I))
                         for wqkv, wo, wgu, wd in self.weights]
        else:
            self.proj = [((lambda x, t=wqkv: F.linear(x, t)), (lambda x, t=wo, residual=None: residual + F.linear(x, t)),
                          (lambda x, gu=wgu, d=wd, residual=None: residual + _bf16_mlp(x, gu, d, I)))
                         for wqkv, wo, wgu, wd in self.weights]
        self.norms = [(torch.ones(H, device=dev, dtype=torch.bfloat16), torch.ones(H, device=dev, dtype=torch.bfloat16))
                      for _ in range(shape.layers)]
        # a prefilled context of `context` positions per sequence (+1 slot for the new token),
        # from its own generator so that a twin sharing `weights` gets the same caches; `kv`
        # shares another model's caches outright
        self.kv = kv if kv is not None else self._make_kv(dev, seed)
        inv = 1.0 / (shape.rope_theta ** (torch.arange(0, hd, 2, device=dev, dtype=torch.float32) / hd))
        ang = context * inv
        # transformers' rotary embedding at the step's position (duplicated halves), per token
        self.cos_full = torch.cat([torch.cos(ang), torch.cos(ang)]).expand(batch, hd).contiguous()
        self.sin_full = torch.cat([torch.sin(ang), torch.sin(ang)]).expand(batch, hd).contiguous()
        self.tokens = torch.zeros(batch, dtype=torch.long, device=dev)
        self.lm_head_int8 = None
        if quantize_lm_head:
            self.set_lm_head_int8(True)

    def _make_kv(self, dev: torch.device, seed: int) -> dict:
        """paged: per layer K and V pools [num_blocks, block_size, H_kv, hd] (the reference's
        layout, plus one spare block as the reference keeps) with a shuffled block table;
        sdpa: per layer contiguous [B, H_kv, context + 1, hd] caches."""
        s, B, hd = self.shape, self.batch, self.shape.head_dim
        gk = torch.Generator(device=dev).manual_seed(seed + 1)
        if self.attention == "sdpa":
            def kv():
                return torch.randn(B, s.kv_heads, self.context + 1, hd, generator=gk, device=dev).to(torch.bfloat16)
            T = self.context + 1  # the new token's slot: position `context` of every sequence
            return {"k": [kv() for _ in range(s.layers)], "v": [kv() for _ in range(s.layers)],
                    "kv_off": (torch.arange(B, device=dev) * s.kv_heads * T + self.context) * hd,
                    "kv_head_stride": T * hd}
        bs = self.block_size
        nbps = -(-(self.context + 1) // bs)
        nb = B * nbps + 1
        gp = torch.Generator().manual_seed(seed + 2)
        table = torch.randperm(nb, generator=gp)[: B * nbps].view(B, nbps).to(torch.int32).to(dev)

        def pool():
            return torch.randn(nb, bs, s.kv_heads, hd, generator=gk, device=dev).to(torch.bfloat16)
        pos = self.context  # the new token's position
        slot = table[:, pos // bs].long() * bs + pos % bs  # its pool slot per sequence
        return {"k": [pool() for _ in range(s.layers)], "v": [pool() for _ in range(s.layers)],
                "block_table": table, "kv_off": slot * s.kv_heads * hd, "kv_head_stride": hd,
                "context_len": torch.full((B,), self.context + 1, dtype=torch.int32, device=dev)}

    def set_lm_head_int8(self, on: bool) -> None:
        """Serve the lm_head (vocab x hidden) from an int8 copy of its weight, or from bf16."""
        self.lm_head_int8 = Int8Linear.from_float_weights(self.lm_head) if on else None

    def _head(self, h: torch.Tensor) -> torch.Tensor:
        return self.lm_head_int8(h) if self.lm_head_int8 is not None else F.linear(h, self.lm_head)

    def layer(self, li: int, h: torch.Tensor, in_place: bool = False) -> torch.Tensor:
        """Decoder layer `li` on the residual stream `h` [B, H]; returns the new stream.
        `in_place` writes the new K/V into the caches (the decode step); otherwise into copies
        (a side-effect-free check)."""
        s = self.shape
        B, hd = self.batch, s.head_dim
        qkv_p, o_p, mlp = self.proj[li]
        n_in, n_post = self.norms[li]
        fused = self.quantize and self.fuse_norms
        if fused and isinstance(qkv_p, Int8Linear):  # RMSNorm straight into the projection's activation planes
            qkv = ops.rms_norm_proj(h, n_in, s.eps, qkv_p.weight_packed, qkv_p.scale, qkv_p.out_features,
                                    qkv_p.in_features)
        else:
            qkv = qkv_p(_rms_norm(h, n_in, s.eps))
        kc, vc = self.kv["k"][li], self.kv["v"][li]
        if not in_place:
            kc, vc = kc.clone(), vc.clone()
        # RoPE on q and k, k and v into their slots, q as (heads, B, hd): one kernel
        qh = ops.rope_kv_write(qkv, s.heads, s.kv_heads, hd, self.cos_full, self.sin_full, kc, vc,
                               self.kv["kv_off"], self.kv["kv_head_stride"])
        q = qh.transpose(0, 1)  # [B, heads, hd] view
        if self.attention == "paged":
            attn = ops.paged_decode_attention(q, kc, vc, self.kv["block_table"], self.kv["context_len"],
                                              self.context + 1)
        else:
            attn = F.scaled_dot_product_attention(q.unsqueeze(2), kc, vc, enable_gqa=True)
        h = o_p(attn.reshape(B, s.heads * hd), residual=h)  # residual + o_proj(attn)
        if fused and isinstance(mlp, Int8LlamaMLP) and mlp._silu():
            g = mlp.gate_up
            act = ops.rms_norm_proj(h, n_post, s.eps, g.weight_packed, g.scale, mlp.intermediate_size, g.in_features,
                                    silu=True)
            return mlp.down_proj(act, residual=h)
        return mlp(_rms_norm(h, n_post, s.eps), residual=h)

    def _hidden(self, tokens: torch.Tensor, in_place: bool, trace: list | None = None) -> torch.Tensor:
        """Final-norm hidden state of one step (`layer` over every layer); `trace`, when
        given, receives each layer's input stream."""
        h = self.embed[tokens]  # [B, H]
        for li in range(self.shape.layers):
            if trace is not None:
                trace.append(h)
            h = self.layer(li, h, in_place)
        return _rms_norm(h, self.final_norm, self.shape.eps)

    def dequantized_weights(self, dtype: torch.dtype = torch.bfloat16) -> list:
        """Per layer the dequantized int8 weights in `weights` order ([q;k;v], o, [gate;up],
        down): the bf16 twin that isolates the int8 kernels' arithmetic."""
        if not self.quantize:
            raise ValueError("dequantized_weights: the model is not quantized")
        return [(qkv.dequantized(dtype), o.dequantized(dtype),
                 torch.cat([mlp.gate_weight(dtype), mlp.up_weight(dtype)]), mlp.down_proj.dequantized(dtype))
                for qkv, o, mlp in self.proj]

    def step(self, tokens: torch.Tensor | None = None) -> torch.Tensor:
        """One decode step for every sequence; returns the greedy next tokens [B]."""
        h = self._hidden(self.tokens if tokens is None else tokens, in_place=True)
        return self._head(h).argmax(-1)

    def logits(self, tokens: torch.Tensor) -> torch.Tensor:
        """fp32 logits of one step, leaving the caches untouched (parity checks)."""
        return self._head(self._hidden(tokens, in_place=False)).float()
