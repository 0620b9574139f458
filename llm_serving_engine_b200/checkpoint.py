"""On-disk int8 checkpoint of the quantized projections.

The reference loads a bf16/fp16 Hugging Face checkpoint (`model_runner.py:50-53`) and, with
int8 selected, this package quantizes every projection on the GPU at load
(`quantize_llama_`).  This module stores the result, so that a later load skips the
quantization and never holds the bf16 projection weights: for Llama-3-70B that is 68 GB of
int8 weights and scales instead of 137 GB of bf16 in host or device memory.

Format: one safetensors file (the container format of Hugging Face checkpoints), tensors
in row-major `[out_features, in_features]` int8 plus fp32 per-row scales, so the file does
not depend on the kernels' in-memory packed layout.  Per decoder layer i, with prefix
`model.layers.{i}.`:

    self_attn.qkv_proj.qweight   int8 [q + k + v, hidden]   (fused [q; k; v] rows)
    self_attn.qkv_proj.scale     fp32 [q + k + v]
    self_attn.o_proj.qweight     int8 [hidden, q]
    self_attn.o_proj.scale       fp32 [hidden]
    mlp.gate_up_proj.qweight     int8 [2 I, hidden]          (fused [gate; up] rows)
    mlp.gate_up_proj.scale       fp32 [2 I]
    mlp.down_proj.qweight        int8 [hidden, I]
    mlp.down_proj.scale          fp32 [hidden]

optionally `lm_head.qweight` int8 [vocab, hidden] with `lm_head.scale` (a model quantized
with `quantize_llama_(..., lm_head=True)`), and string metadata: `format`
(`lse-int8-per-channel`), `version`, `num_layers`, `qkv_sizes` (`q,k,v`) and
`intermediate_size`.  The quantization rule is the one
`ops.quantize_per_channel` applies: s = max|w|/127 per row (1.0 for a zero row),
q = clamp(rint(w/s), -127, 127).

`read_int8_checkpoint` / `write_int8_checkpoint` are the file layer (CPU only);
`save_int8_checkpoint(model, path)` takes a model after `quantize_llama_`, and
`load_int8_checkpoint_(model, path)` installs the same int8 modules `quantize_llama_` would,
from the file, into a Llama-family model whose projection weights are never read (they may
live on the meta device).
"""

from __future__ import annotations

import torch
import torch.nn as nn

FORMAT = "lse-int8-per-channel"
VERSION = "1"
FILE_NAME = "int8_projections.safetensors"

_PROJ = ("self_attn.qkv_proj", "self_attn.o_proj", "mlp.gate_up_proj", "mlp.down_proj")

__all__ = ["FORMAT", "VERSION", "FILE_NAME", "write_int8_checkpoint", "read_int8_checkpoint",
           "int8_state_dict", "save_int8_checkpoint", "load_int8_checkpoint_"]


def _key(layer: int, proj: str, part: str) -> str:
    return f"model.layers.{layer}.{proj}.{part}"


def _check_tensors(tensors: dict[str, torch.Tensor], meta: dict[str, str]) -> tuple[int, tuple[int, int, int], int]:
    """Validate a checkpoint's tensors against its metadata; returns (layers, qkv sizes, I)."""
    if meta.get("format") != FORMAT:
        raise ValueError(f"int8 checkpoint: format {meta.get('format')!r}, expected {FORMAT!r}")
    if meta.get("version") != VERSION:
        raise ValueError(f"int8 checkpoint: version {meta.get('version')!r}, expected {VERSION!r}")
    try:
        layers = int(meta["num_layers"])
        sizes = tuple(int(v) for v in meta["qkv_sizes"].split(","))
        inter = int(meta["intermediate_size"])
    except (KeyError, ValueError) as e:
        raise ValueError(f"int8 checkpoint: bad metadata ({e})") from None
    if len(sizes) != 3 or layers < 1 or inter < 1:
        raise ValueError("int8 checkpoint: bad metadata (qkv_sizes, num_layers, intermediate_size)")
    expected = {_key(i, p, part) for i in range(layers) for p in _PROJ for part in ("qweight", "scale")}
    head = {"lm_head.qweight", "lm_head.scale"}
    if head & set(tensors):
        expected |= head
    if set(tensors) != expected:
        missing, extra = sorted(expected - set(tensors)), sorted(set(tensors) - expected)
        raise ValueError(f"int8 checkpoint: missing {missing[:4]}, unexpected {extra[:4]}")
    hidden = None
    for i in range(layers):
        rows = {"self_attn.qkv_proj": sum(sizes), "mlp.gate_up_proj": 2 * inter}
        for p in _PROJ:
            q, s = tensors[_key(i, p, "qweight")], tensors[_key(i, p, "scale")]
            if q.dtype != torch.int8 or q.dim() != 2 or s.dtype != torch.float32 or s.shape != (q.shape[0],):
                raise ValueError(f"int8 checkpoint: {_key(i, p, '*')} must be int8 [N, K] with fp32 [N] scales")
            if p in rows and q.shape[0] != rows[p]:
                raise ValueError(f"int8 checkpoint: {_key(i, p, 'qweight')} has {q.shape[0]} rows, expected {rows[p]}")
        hidden = tensors[_key(i, "self_attn.qkv_proj", "qweight")].shape[1] if hidden is None else hidden
        if (tensors[_key(i, "self_attn.o_proj", "qweight")].shape != (hidden, sizes[0])
                or tensors[_key(i, "mlp.gate_up_proj", "qweight")].shape[1] != hidden
                or tensors[_key(i, "mlp.down_proj", "qweight")].shape != (hidden, inter)):
            raise ValueError(f"int8 checkpoint: layer {i} projection shapes do not chain")
    if "lm_head.qweight" in tensors:
        q, s = tensors["lm_head.qweight"], tensors["lm_head.scale"]
        if (q.dtype != torch.int8 or q.dim() != 2 or q.shape[1] != hidden or s.dtype != torch.float32
                or s.shape != (q.shape[0],)):
            raise ValueError("int8 checkpoint: lm_head must be int8 [vocab, hidden] with fp32 [vocab] scales")
    return layers, sizes, inter


def write_int8_checkpoint(path: str, tensors: dict[str, torch.Tensor], meta: dict[str, str]) -> None:
    """Write validated int8 projection tensors (any device) and their metadata to `path`."""
    from safetensors.torch import save_file

    meta = {"format": FORMAT, "version": VERSION, **{k: str(v) for k, v in meta.items()}}
    _check_tensors(tensors, meta)
    save_file({k: v.detach().contiguous().cpu() for k, v in tensors.items()}, path, metadata=meta)


def read_int8_checkpoint(path: str, device: str | torch.device = "cpu"
                         ) -> tuple[dict[str, torch.Tensor], dict[str, str]]:
    """Read and validate an int8 checkpoint; tensors land on `device`."""
    from safetensors import safe_open

    with safe_open(path, framework="pt", device=str(device)) as f:
        meta = dict(f.metadata() or {})
        tensors = {k: f.get_tensor(k) for k in f.keys()}
    _check_tensors(tensors, meta)
    return tensors, meta


def _layers(model: nn.Module):
    decoder = getattr(model, "model", model)
    layers = getattr(decoder, "layers", None)
    if layers is None:
        raise RuntimeError(f"int8 checkpoint: {type(model).__name__} has no Llama-family decoder layers")
    return layers


def int8_state_dict(model: nn.Module) -> tuple[dict[str, torch.Tensor], dict[str, str]]:
    """The int8 projections of a model after `quantize_llama_` (fused or not), as row-major
    int8 weights and fp32 scales in the checkpoint's key layout, plus its metadata."""
    from .int8_linear import FusedInt8QKV, Int8Linear, Int8LlamaMLP

    tensors: dict[str, torch.Tensor] = {}
    sizes = inter = None
    for i, layer in enumerate(_layers(model)):
        attn, mlp = layer.self_attn, layer.mlp
        qkv = getattr(attn, "qkv_int8", None)
        if isinstance(qkv, FusedInt8QKV):
            q, s, sz = qkv.fused.weight, qkv.fused.scale, qkv.sizes
        elif all(isinstance(getattr(attn, n), Int8Linear) for n in ("q_proj", "k_proj", "v_proj")):
            parts = [getattr(attn, n) for n in ("q_proj", "k_proj", "v_proj")]
            q = torch.cat([p.weight for p in parts])
            s = torch.cat([p.scale for p in parts])
            sz = tuple(p.out_features for p in parts)
        else:
            raise RuntimeError(f"int8 checkpoint: layer {i} attention is not quantized (run quantize_llama_ first)")
        if not isinstance(attn.o_proj, Int8Linear) or not isinstance(mlp, Int8LlamaMLP):
            raise RuntimeError(f"int8 checkpoint: layer {i} is not quantized (run quantize_llama_ first)")
        if sizes is not None and (tuple(sz) != sizes or mlp.intermediate_size != inter):
            raise RuntimeError("int8 checkpoint: layers of different shapes are not supported")
        sizes, inter = tuple(sz), mlp.intermediate_size
        g, u = mlp.split_rows(mlp.gate_up.weight)
        gs, us = mlp.split_rows(mlp.gate_up.scale)
        tensors[_key(i, "self_attn.qkv_proj", "qweight")] = q
        tensors[_key(i, "self_attn.qkv_proj", "scale")] = s
        tensors[_key(i, "self_attn.o_proj", "qweight")] = attn.o_proj.weight
        tensors[_key(i, "self_attn.o_proj", "scale")] = attn.o_proj.scale
        tensors[_key(i, "mlp.gate_up_proj", "qweight")] = torch.cat([g, u])
        tensors[_key(i, "mlp.gate_up_proj", "scale")] = torch.cat([gs, us])
        tensors[_key(i, "mlp.down_proj", "qweight")] = mlp.down_proj.weight
        tensors[_key(i, "mlp.down_proj", "scale")] = mlp.down_proj.scale
    head = getattr(model, "lm_head", None)
    if isinstance(head, Int8Linear):
        tensors["lm_head.qweight"] = head.weight
        tensors["lm_head.scale"] = head.scale
    meta = {"num_layers": str(len(_layers(model))), "qkv_sizes": ",".join(map(str, sizes)),
            "intermediate_size": str(inter)}
    return tensors, meta


def save_int8_checkpoint(model: nn.Module, path: str) -> None:
    """Write the int8 projections of a quantized model (`quantize_llama_`) to `path`."""
    tensors, meta = int8_state_dict(model)
    write_int8_checkpoint(path, tensors, meta)


@torch.no_grad()
def load_int8_checkpoint_(model: nn.Module, path: str, device: str | torch.device | None = None,
                          fuse: bool = True) -> nn.Module:
    """In place: install the int8 projections stored at `path` into `model` (the modules
    `quantize_llama_(model, fuse)` installs), without reading the model's own projection
    weights.  `device` defaults to the device of the model's embedding (a CUDA device)."""
    from .int8_linear import FusedInt8QKV, Int8Linear, Int8LlamaMLP

    layers = _layers(model)
    if device is None:
        emb = model.get_input_embeddings() if hasattr(model, "get_input_embeddings") else None
        device = emb.weight.device if emb is not None else torch.device("cuda")
    device = torch.device(device)
    if device.type != "cuda":
        raise RuntimeError("int8 checkpoint: the int8 modules run on CUDA only (no CPU fallback)")
    tensors, meta = read_int8_checkpoint(path, device=device)
    n_layers, sizes, inter = _check_tensors(tensors, meta)
    if n_layers != len(layers):
        raise ValueError(f"int8 checkpoint: {n_layers} layers in the file, {len(layers)} in the model")
    for i, layer in enumerate(layers):
        attn = layer.self_attn
        want = (attn.q_proj.out_features, attn.k_proj.out_features, attn.v_proj.out_features)
        if want != sizes or layer.mlp.down_proj.in_features != inter:
            raise ValueError(f"int8 checkpoint: layer {i} shapes {sizes}, I={inter} do not match the model {want}")
        q, s = tensors.pop(_key(i, "self_attn.qkv_proj", "qweight")), tensors.pop(_key(i, "self_attn.qkv_proj", "scale"))
        if fuse:
            qkv = FusedInt8QKV(Int8Linear.from_quantized(q, s), sizes)
            attn.qkv_int8 = qkv
            attn.q_proj, attn.k_proj, attn.v_proj = qkv.facades()
        else:
            offs = [0, sizes[0], sizes[0] + sizes[1], sum(sizes)]
            attn.q_proj, attn.k_proj, attn.v_proj = (
                Int8Linear.from_quantized(q[offs[j]:offs[j + 1]], s[offs[j]:offs[j + 1]]) for j in range(3))
        attn.o_proj = Int8Linear.from_quantized(tensors.pop(_key(i, "self_attn.o_proj", "qweight")),
                                                tensors.pop(_key(i, "self_attn.o_proj", "scale")))
        act = getattr(layer.mlp, "act_fn", None)
        layer.mlp = Int8LlamaMLP.from_quantized(
            tensors.pop(_key(i, "mlp.gate_up_proj", "qweight")), tensors.pop(_key(i, "mlp.gate_up_proj", "scale")),
            tensors.pop(_key(i, "mlp.down_proj", "qweight")), tensors.pop(_key(i, "mlp.down_proj", "scale")),
            inter, **({"act": act} if act is not None else {}))
    if "lm_head.qweight" in tensors:
        head = getattr(model, "lm_head", None)
        if head is None or head.in_features != tensors["lm_head.qweight"].shape[1] or \
                head.out_features != tensors["lm_head.qweight"].shape[0]:
            raise ValueError("int8 checkpoint: the stored lm_head does not match the model's")
        model.lm_head = Int8Linear.from_quantized(tensors.pop("lm_head.qweight"), tensors.pop("lm_head.scale"))
    torch.cuda.empty_cache()
    return model
