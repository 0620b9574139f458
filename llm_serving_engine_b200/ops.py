"""Torch-facing int8 linear ops over the C ABI (liblse_int8.so).

`int8_linear(x, weight, scale)` is the call every int8 projection makes: the replacement
for `torch.nn.Linear.__call__` at the reference's call sites
(`src/llm_serving_engine/model/model_runner.py:322-324`, `:369`, `:418`, `:223`;
`src/llm_serving_engine/model/piecewise_graph.py:163-166`).  Shapes, dtypes and devices are
validated on the host and raise `ValueError` / `RuntimeError` before anything launches, the
way the reference surfaces load-time refusals (`model_runner.py:77-94`).

Graph capture: the op launches on `torch.cuda.current_stream()`, never synchronizes and
never allocates outside the torch caching allocator, so the reference's decode and piecewise
CUDA-graph captures (`decode_graph.py:87-116`, `piecewise_graph.py:71-109`) record it like
any other kernel.  The tensor-core path's scratch (stream-K counters and partial tiles, the
activation digit planes) is taken from the caching allocator on every call, like the
output: the library initialises what it uses, so the block may be any earlier tensor's, on
any stream, inside a capture or not, and nothing persists between calls.
"""

from __future__ import annotations

import threading

import torch

from . import _lib

__all__ = [
    "torch_ops",
    "int8_linear",
    "int8_linear_packed",
    "pack_weight",
    "unpack_weight",
    "packed_weight_bytes",
    "quantize_per_channel",
    "interleave_gate_up_rows",
    "int8_gate_up_silu_packed",
    "GATE_UP_SILU_MAX_M",
    "paged_decode_attention",
    "paged_attention",
    "set_wait_limit",
    "rope_kv_write",
    "rms_norm", "rms_norm_proj",
    "pool_slot_offsets",
    "linear_workspace",
    "device_status",
    "ALGO_AUTO",
    "ALGO_GEMV",
    "ALGO_TCGEN05",
    "ALGO_SKINNY",
]

ALGO_AUTO = _lib.ALGO_AUTO
ALGO_GEMV = _lib.ALGO_GEMV
ALGO_TCGEN05 = _lib.ALGO_TCGEN05
ALGO_SKINNY = _lib.ALGO_SKINNY

_DTYPE_CODES = {torch.bfloat16: _lib.DT_BF16, torch.float16: _lib.DT_F16, torch.float32: _lib.DT_F32}

_inited: set[int] = set()
_ws_lock = threading.Lock()
_torch_ops_lock = threading.Lock()
_torch_ops_loaded = False


def torch_ops():
    """`torch.ops.lse` with `int8_linear` and `gate_up_silu` registered (liblse_torch.so, the
    C++ operators over the C ABI: one dispatcher call per projection).  Built in-tree on first
    use if missing."""
    global _torch_ops_loaded
    if not _torch_ops_loaded:
        with _torch_ops_lock:
            if not _torch_ops_loaded:
                import os

                from . import build as _build

                _lib.load()  # the C ABI library the operators link to, built if missing
                path = _build.TORCH_LIB_PATH
                if not os.path.exists(path):
                    _build.build_torch_ops()
                torch.ops.load_library(path)
                _torch_ops_loaded = True
    return torch.ops.lse


def _ensure_device(device: torch.device) -> None:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx not in _inited:
        _lib.check(_lib.load().lse_init(idx), f"lse_init(cuda:{idx})")
        _inited.add(idx)


def linear_workspace(M: int, K: int, N: int, device: torch.device, algo: int = _lib.ALGO_AUTO,
                     packed: bool = True) -> torch.Tensor | None:
    """Scratch for one call (None when the chosen kernel needs none): a fresh block of the
    torch caching allocator on the current stream, its contents irrelevant to the library."""
    nbytes = int(_lib.load().lse_int8_linear_workspace_for(M, K, N, int(algo), 1 if packed else 0))
    if nbytes == 0:
        return None
    return torch.empty(nbytes, dtype=torch.uint8, device=device)


def _check_x(x: torch.Tensor, K: int, *tensors: torch.Tensor) -> None:
    if not (x.is_cuda and all(t.is_cuda for t in tensors)):
        raise RuntimeError("int8_linear runs on CUDA only (no CPU fallback)")
    if any(t.device != x.device for t in tensors):
        raise ValueError(f"int8_linear: tensors on different devices ({x.device}, {[t.device for t in tensors]})")
    if x.dtype not in (torch.bfloat16, torch.float16):
        raise ValueError(f"int8_linear: x must be bfloat16 or float16, got {x.dtype}")
    if x.shape[-1] != K:
        raise ValueError(f"int8_linear: x last dim {x.shape[-1]} != in_features {K}")
    if K % 16 != 0:
        raise ValueError(f"int8_linear: in_features must be a multiple of 16, got {K}")


def _launch(x: torch.Tensor, w_ptr: int, scale: torch.Tensor, N: int, K: int, out, algo: int, packed: bool,
            residual: torch.Tensor | None = None):
    lead = x.shape[:-1]
    x2 = x.reshape(-1, K)
    if x2.stride(-1) != 1 or x2.stride(0) % 8 != 0 or x2.data_ptr() % 16 != 0:
        x2 = x2.contiguous()
    M = x2.shape[0]
    if not packed and x.dtype != torch.bfloat16:
        raise ValueError("int8_linear: row-major weights take bf16 activations (fp16: the packed layout)")
    if out is None:
        y2 = torch.empty((M, N), dtype=x.dtype, device=x.device)
        y = y2.view(*lead, N)
    else:
        if out.dtype != x.dtype or out.shape != (*lead, N) or out.stride(-1) != 1:
            raise ValueError("int8_linear: out must be [..., N] of x's dtype with a contiguous last dim")
        y = out
        y2 = out.view(-1, N) if M > 0 else out.reshape(0, N)
    r2 = None
    if residual is not None:
        if (residual.dtype != x.dtype or residual.device != x.device or residual.shape != (*lead, N)
                or residual.stride(-1) != 1):
            raise ValueError("int8_linear: residual must be [..., N] of x's dtype and device with a contiguous last dim")
        r2 = residual.view(-1, N) if M > 0 else None
    if M == 0:
        return y
    _ensure_device(x.device)
    stream = torch.cuda.current_stream(x.device)
    ws = linear_workspace(M, K, N, x.device, algo, packed)
    ws_ptr, ws_bytes = (ws.data_ptr(), ws.numel()) if ws is not None else (None, 0)
    lib = _lib.load()
    if r2 is not None and r2.data_ptr() == y2.data_ptr() and r2.stride(0) != y2.stride(0):
        raise ValueError("int8_linear: residual and out overlap with different strides")
    if packed:
        rc = lib.lse_int8_linear_packed_dt(x2.data_ptr(), _DTYPE_CODES[x.dtype], M, K, x2.stride(0), w_ptr,
                                           scale.data_ptr(), N, r2.data_ptr() if r2 is not None else None,
                                           r2.stride(0) if r2 is not None else 0, y2.data_ptr(), y2.stride(0),
                                           ws_ptr, ws_bytes, int(algo), stream.cuda_stream)
        _lib.check(rc, "lse_int8_linear_packed_dt")
        return y
    if r2 is not None:
        raise ValueError("int8_linear: the residual add needs the packed weight layout")
    rc = lib.lse_int8_linear_ex(x2.data_ptr(), M, K, x2.stride(0), w_ptr, scale.data_ptr(), N, y2.data_ptr(),
                                y2.stride(0), ws_ptr, ws_bytes, int(algo), stream.cuda_stream)
    _lib.check(rc, "lse_int8_linear")
    return y


def int8_linear(x: torch.Tensor, weight: torch.Tensor, scale: torch.Tensor,
                out: torch.Tensor | None = None, algo: int = ALGO_AUTO) -> torch.Tensor:
    """y = bf16(x @ (weight * scale[:, None]).T): x bf16 [..., K] on CUDA, weight int8 [N, K]
    contiguous (row-major), scale fp32 [N].  Returns bf16 [..., N] (or writes `out`, a
    [..., N] bf16 tensor whose last dim is contiguous)."""
    if weight.dtype != torch.int8 or weight.dim() != 2:
        raise ValueError(f"int8_linear: weight must be int8 [N, K], got {weight.dtype} {tuple(weight.shape)}")
    N, K = weight.shape
    _check_x(x, K, weight, scale)
    if scale.dtype != torch.float32 or scale.shape != (N,):
        raise ValueError(f"int8_linear: scale must be float32 [{N}], got {scale.dtype} {tuple(scale.shape)}")
    if not weight.is_contiguous():
        raise ValueError("int8_linear: weight must be contiguous [N, K]")
    return _launch(x, weight.data_ptr(), scale, N, K, out, algo, packed=False)


def packed_weight_bytes(N: int, K: int) -> int:
    return int(_lib.load().lse_int8_packed_weight_bytes(N, K))


def pack_weight(q: torch.Tensor) -> torch.Tensor:
    """int8 [N, K] (CUDA) -> the tile-contiguous packed layout (1-D int8), once at load."""
    if not q.is_cuda or q.dtype != torch.int8 or q.dim() != 2:
        raise ValueError("pack_weight: need a CUDA int8 [N, K] tensor")
    if q.stride(1) != 1:
        q = q.contiguous()
    N, K = q.shape
    out = torch.empty(packed_weight_bytes(N, K), dtype=torch.int8, device=q.device)
    _ensure_device(q.device)
    rc = _lib.load().lse_int8_pack_weight(q.data_ptr(), N, K, q.stride(0), out.data_ptr(),
                                          torch.cuda.current_stream(q.device).cuda_stream)
    _lib.check(rc, "lse_int8_pack_weight")
    return out


def unpack_weight(packed: torch.Tensor, N: int, K: int) -> torch.Tensor:
    out = torch.empty((N, K), dtype=torch.int8, device=packed.device)
    _ensure_device(packed.device)
    rc = _lib.load().lse_int8_unpack_weight(packed.data_ptr(), N, K, out.data_ptr(),
                                            torch.cuda.current_stream(packed.device).cuda_stream)
    _lib.check(rc, "lse_int8_unpack_weight")
    return out


def int8_linear_packed(x: torch.Tensor, w_packed: torch.Tensor, scale: torch.Tensor, N: int, K: int,
                       out: torch.Tensor | None = None, algo: int = ALGO_AUTO,
                       residual: torch.Tensor | None = None) -> torch.Tensor:
    """int8_linear with the weight in the packed layout (`pack_weight`).  With `residual`
    (bf16 [..., N]) the result is bf16(residual + x @ (W * s).T), rounded once; `residual`
    may be `out` itself (an in-place residual update)."""
    _check_x(x, K, w_packed, scale)
    if w_packed.dtype != torch.int8 or w_packed.numel() != packed_weight_bytes(N, K) or not w_packed.is_contiguous():
        raise ValueError(f"int8_linear_packed: w_packed must be the contiguous packed int8 buffer of [{N}, {K}]")
    if scale.dtype != torch.float32 or scale.shape != (N,):
        raise ValueError(f"int8_linear_packed: scale must be float32 [{N}]")
    return _launch(x, w_packed.data_ptr(), scale, N, K, out, algo, packed=True, residual=residual)


GATE_UP_SILU_MAX_M = _lib.GATE_UP_SILU_MAX_M


def interleave_gate_up_rows(intermediate: int, device=None) -> torch.Tensor:
    """Row order of a fused [gate; up] weight (2 * intermediate rows) that interleaves 8-row
    blocks: gate rows 8j..8j+7, then up rows 8j..8j+7, for every j (the layout
    `int8_gate_up_silu_packed` reads: one 16-row block of the packed weight holds a gate row
    and its up row in the same lane's accumulator)."""
    if intermediate % 8:
        raise ValueError(f"gate/up interleave: intermediate size {intermediate} is not a multiple of 8")
    blk = torch.arange(intermediate, device=device).view(-1, 8)
    return torch.stack([blk, blk + intermediate], dim=1).reshape(-1)


def int8_gate_up_silu_packed(x: torch.Tensor, w_packed: torch.Tensor, scale: torch.Tensor, intermediate: int,
                             K: int, out: torch.Tensor | None = None) -> torch.Tensor:
    """`silu(x @ (Wg * sg).T) * (x @ (Wu * su).T)` in one kernel: the decode kernel for up to
    GATE_UP_SILU_MAX_M tokens, the tensor-core kernel with SiLU * mul in its epilogue above.
    `w_packed` is the packed layout of the gate/up rows in `interleave_gate_up_rows` order,
    `scale` the scales in the same order; returns bf16 [..., intermediate]."""
    _check_x(x, K, w_packed, scale)
    I = intermediate
    if w_packed.dtype != torch.int8 or w_packed.numel() != packed_weight_bytes(2 * I, K) or not w_packed.is_contiguous():
        raise ValueError(f"int8_gate_up_silu_packed: w_packed must be the packed int8 buffer of [{2 * I}, {K}]")
    if scale.dtype != torch.float32 or scale.shape != (2 * I,):
        raise ValueError(f"int8_gate_up_silu_packed: scale must be float32 [{2 * I}]")
    lead = x.shape[:-1]
    x2 = x.reshape(-1, K)
    if x2.stride(-1) != 1 or x2.stride(0) % 8 != 0 or x2.data_ptr() % 16 != 0:
        x2 = x2.contiguous()
    M = x2.shape[0]
    if out is None:
        out = torch.empty((*lead, I), dtype=x.dtype, device=x.device)
    elif out.dtype != x.dtype or out.shape != (*lead, I) or not out.is_contiguous():
        raise ValueError("int8_gate_up_silu_packed: out must be contiguous [..., intermediate] of x's dtype")
    if M == 0:
        return out
    _ensure_device(x.device)
    stream = torch.cuda.current_stream(x.device)
    # above the decode kernel's range the fused entry always runs the tensor-core kernel
    ws = linear_workspace(M, K, 2 * I, x.device, _lib.ALGO_TCGEN05) if M > GATE_UP_SILU_MAX_M else None
    ws_ptr, ws_bytes = (ws.data_ptr(), ws.numel()) if ws is not None else (None, 0)
    rc = _lib.load().lse_int8_gate_up_silu_packed_dt(x2.data_ptr(), _DTYPE_CODES[x.dtype], M, K, x2.stride(0),
                                                     w_packed.data_ptr(), scale.data_ptr(), I, out.data_ptr(), I,
                                                     ws_ptr, ws_bytes, stream.cuda_stream)
    _lib.check(rc, "lse_int8_gate_up_silu_packed_dt")
    return out


def quantize_per_channel(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Symmetric per-output-channel int8 quantization of a CUDA weight [N, K] (bf16, fp16 or
    fp32): s = max|w[n,:]|/127 (1.0 for an all-zero row), q = clamp(rint(w/s), -127, 127)."""
    if not w.is_cuda:
        raise RuntimeError("quantize_per_channel runs on CUDA only (no CPU fallback)")
    if w.dim() != 2 or w.dtype not in _DTYPE_CODES:
        raise ValueError(f"quantize_per_channel: need a 2-D bf16/fp16/fp32 weight, got {w.dtype} {tuple(w.shape)}")
    if w.stride(1) != 1:
        w = w.contiguous()
    N, K = w.shape
    q = torch.empty((N, K), dtype=torch.int8, device=w.device)
    s = torch.empty((N,), dtype=torch.float32, device=w.device)
    if N == 0:
        return q, s
    _ensure_device(w.device)
    stream = torch.cuda.current_stream(w.device)
    rc = _lib.load().lse_int8_quantize(w.data_ptr(), _DTYPE_CODES[w.dtype], N, K, w.stride(0),
                                       q.data_ptr(), s.data_ptr(), stream.cuda_stream)
    _lib.check(rc, "lse_int8_quantize")
    return q, s


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float, out: torch.Tensor | None = None) -> torch.Tensor:
    """transformers' LlamaRMSNorm on bf16 or fp16 rows in one kernel: x [..., N] (last dim
    contiguous), weight [N] of x's dtype; fp32 arithmetic with the module's two roundings."""
    if x.dtype not in (torch.bfloat16, torch.float16) or weight.dtype != x.dtype or not (x.is_cuda and weight.is_cuda):
        raise ValueError("rms_norm: x and weight must be bf16 or fp16 CUDA tensors of one dtype")
    N = x.shape[-1]
    if weight.shape != (N,) or not weight.is_contiguous():
        raise ValueError(f"rms_norm: weight must be contiguous [{N}]")
    x2 = x.reshape(-1, N)
    if x2.stride(-1) != 1 or x2.stride(0) % 8 or x2.data_ptr() % 16:
        x2 = x2.contiguous()
    if out is None:
        out = torch.empty(x.shape, dtype=x.dtype, device=x.device)
    elif out.dtype != x.dtype or out.shape != x.shape or not out.is_contiguous():
        raise ValueError("rms_norm: out must be a contiguous tensor of x's shape and dtype")
    y2 = out.view(-1, N)
    if x2.shape[0] == 0:
        return out
    _ensure_device(x.device)
    rc = _lib.load().lse_rms_norm_dt(x2.data_ptr(), _DTYPE_CODES[x.dtype], x2.shape[0], N, x2.stride(0),
                                     weight.data_ptr(), float(eps), y2.data_ptr(), y2.stride(0),
                                     torch.cuda.current_stream(x.device).cuda_stream)
    _lib.check(rc, "lse_rms_norm_dt")
    return out


def rms_norm_proj(x: torch.Tensor, norm_weight: torch.Tensor, eps: float, w_packed: torch.Tensor, scale: torch.Tensor,
                  N: int, K: int, silu: bool = False, out: torch.Tensor | None = None) -> torch.Tensor:
    """The packed projection of `rms_norm(x, norm_weight, eps)` in one call, bf16: with
    silu=False `int8_linear_packed(rms_norm(x), w_packed, scale, N, K)` ([..., N]); with
    silu=True `int8_gate_up_silu_packed(rms_norm(x), w_packed, scale, N, K)` ([..., N], the
    weight holding 2N interleaved gate/up rows).  Bitwise the same as those two calls; where the
    projection takes the tensor-core kernel the normalisation writes its digit planes directly."""
    _check_x(x, K, norm_weight, w_packed, scale)
    if x.dtype != torch.bfloat16 or norm_weight.dtype != torch.bfloat16 or norm_weight.shape != (K,) \
            or not norm_weight.is_contiguous():
        raise ValueError(f"rms_norm_proj: x must be bf16 and norm_weight contiguous bf16 [{K}]")
    rows = 2 * N if silu else N
    if w_packed.dtype != torch.int8 or w_packed.numel() != packed_weight_bytes(rows, K) or not w_packed.is_contiguous():
        raise ValueError(f"rms_norm_proj: w_packed must be the packed int8 buffer of [{rows}, {K}]")
    if scale.dtype != torch.float32 or scale.shape != (rows,):
        raise ValueError(f"rms_norm_proj: scale must be float32 [{rows}]")
    lead = x.shape[:-1]
    x2 = x.reshape(-1, K)
    if x2.stride(-1) != 1 or x2.stride(0) % 8 != 0 or x2.data_ptr() % 16 != 0:
        x2 = x2.contiguous()
    M = x2.shape[0]
    if out is None:
        out = torch.empty((*lead, N), dtype=x.dtype, device=x.device)
    elif out.dtype != x.dtype or out.shape != (*lead, N) or not out.is_contiguous():
        raise ValueError("rms_norm_proj: out must be contiguous [..., N] bf16")
    if M == 0:
        return out
    _ensure_device(x.device)
    lib = _lib.load()
    ws = torch.empty(int(lib.lse_int8_rms_norm_proj_workspace(M, K)), dtype=torch.uint8, device=x.device)
    fn = lib.lse_int8_rms_norm_gate_up_silu_packed if silu else lib.lse_int8_rms_norm_linear_packed
    rc = fn(x2.data_ptr(), M, K, x2.stride(0), norm_weight.data_ptr(), float(eps), w_packed.data_ptr(), scale.data_ptr(),
            N, out.data_ptr(), N, ws.data_ptr(), ws.numel(), torch.cuda.current_stream(x.device).cuda_stream)
    _lib.check(rc, "lse_int8_rms_norm_gate_up_silu_packed" if silu else "lse_int8_rms_norm_linear_packed")
    return out


def pool_slot_offsets(dest_block_id: torch.Tensor, dest_within: torch.Tensor, k_pool: torch.Tensor) -> torch.Tensor:
    """int64 element offsets of tokens' slots (KV head 0) in a [num_blocks, block_size, H_kv, D]
    pool, from the reference's `dest_block_id` / `dest_within` (`model_runner.py:342-355`)."""
    _nb, bs, h_kv, d = k_pool.shape
    return (dest_block_id.long() * bs + dest_within.long()) * (h_kv * d)


def rope_kv_write(qkv: torch.Tensor, n_heads: int, n_kv_heads: int, head_dim: int, cos: torch.Tensor,
                  sin: torch.Tensor, k_dst: torch.Tensor, v_dst: torch.Tensor, kv_offset: torch.Tensor,
                  kv_head_stride: int | None = None, q_out: torch.Tensor | None = None) -> torch.Tensor:
    """RoPE on q and k of the fused QKV output, k and v written to their slots, q returned as
    (n_heads, tokens, head_dim) - `write_kv_and_project_q` after the projection, in one launch.

    qkv: bf16 or fp16 [M, (H + 2 H_kv) * D] (last dim contiguous); cos / sin: [M, D] fp32, bf16
    or fp16 (transformers' per-token rotary embedding, duplicated halves); k_dst / v_dst: caches
    of qkv's dtype
    (e.g. the [num_blocks, block_size, H_kv, D] pools); kv_offset: int64 [M] element offsets
    of each token's slot for KV head 0 (`pool_slot_offsets`), KV heads kv_head_stride apart
    (default head_dim).
    """
    M = qkv.shape[0]
    D = head_dim
    dt = qkv.dtype
    if dt not in (torch.bfloat16, torch.float16) or qkv.dim() != 2 or qkv.stride(-1) != 1 \
            or qkv.shape[1] != (n_heads + 2 * n_kv_heads) * D:
        raise ValueError("rope_kv_write: qkv must be bf16 or fp16 [M, (H + 2 H_kv) * D] with a contiguous last dim")
    if cos.shape != (M, D) or sin.shape != (M, D) or cos.dtype != sin.dtype or cos.stride() != sin.stride() \
            or cos.stride(-1) != 1 or cos.dtype not in (torch.float32, torch.bfloat16, torch.float16):
        raise ValueError("rope_kv_write: cos / sin must be [M, D] fp32, bf16 or fp16 with equal, row-contiguous strides")
    if k_dst.dtype != dt or v_dst.dtype != dt or not (k_dst.is_contiguous() and v_dst.is_contiguous()):
        raise ValueError("rope_kv_write: k_dst / v_dst must be contiguous, of qkv's dtype")
    if kv_offset.dtype != torch.int64 or kv_offset.shape != (M,) or not kv_offset.is_contiguous():
        raise ValueError("rope_kv_write: kv_offset must be int64 [M]")
    if not all(t.is_cuda and t.device == qkv.device for t in (cos, sin, k_dst, v_dst, kv_offset)):
        raise RuntimeError("rope_kv_write runs on CUDA only, all tensors on qkv's device")
    if q_out is None:
        q_out = torch.empty((n_heads, M, D), dtype=dt, device=qkv.device)
    elif q_out.dtype != dt or q_out.shape != (n_heads, M, D) or not q_out.is_contiguous():
        raise ValueError("rope_kv_write: q_out must be contiguous [H, M, D] of qkv's dtype")
    if M == 0:
        return q_out
    _ensure_device(qkv.device)
    cs = _DTYPE_CODES[cos.dtype]
    rc = _lib.load().lse_rope_kv_write_dt(
        qkv.data_ptr(), _DTYPE_CODES[dt], M, qkv.stride(0), n_heads, n_kv_heads, D, cos.data_ptr(), sin.data_ptr(),
        cos.stride(0), cs,
        q_out.data_ptr(), k_dst.data_ptr(), v_dst.data_ptr(), kv_offset.data_ptr(),
        D if kv_head_stride is None else int(kv_head_stride), torch.cuda.current_stream(qkv.device).cuda_stream)
    _lib.check(rc, "lse_rope_kv_write_dt")
    return q_out


# Split-K scratch of the decode attention: one zero-initialised, grow-only buffer per (device,
# stream); its arrival counters sit at a fixed place for every launch shape and every call
# leaves them at zero.  Created (or grown) outside captures only.
_attn_ws: dict[tuple, torch.Tensor] = {}
_attn_ws_retired: list[torch.Tensor] = []  # outgrown buffers stay alive: captured graphs may use them


def paged_decode_attention(q: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor, block_table: torch.Tensor,
                           context_len: torch.Tensor, max_context: int, scale: float | None = None,
                           out: torch.Tensor | None = None, split: bool = True) -> torch.Tensor:
    """Decode attention over the paged K/V pool: one query token per sequence.

    q: bf16 [E, H, D] (d contiguous); k_pool / v_pool: bf16 [num_blocks, block_size, H_KV, D]
    contiguous (the reference's per-layer pool, already holding this step's K/V);
    block_table: int32 [E, >= ceil(max_context / block_size)]; context_len: int32 [E], every
    entry <= max_context (a launch-shape bound, fixed per captured graph).  Returns bf16
    [E, H, D] = softmax(q K^T * scale) V over each sequence's positions, scale = 1/sqrt(D) by
    default (`paged_attention_forward`, `kernels/flash_attention.py:287-332`, with q_len 1).
    split=False runs one CTA per (sequence, KV head) with no workspace (nothing to size or keep
    per stream; any max_context, a sequence's first 1024 blocks of positions covered, a longer
    context reported as LSE_ERR_UNSUPPORTED on the status word).
    """
    if not all(t.is_cuda for t in (q, k_pool, v_pool, block_table, context_len)):
        raise RuntimeError("paged_decode_attention runs on CUDA only (no CPU fallback)")
    if q.dtype not in (torch.bfloat16, torch.float16) or k_pool.dtype != q.dtype or v_pool.dtype != q.dtype:
        raise ValueError("paged_decode_attention: q and the pools must be bfloat16 or float16, of one dtype")
    if q.dim() != 3 or q.stride(-1) != 1:
        raise ValueError("paged_decode_attention: q must be [E, H, D] with a contiguous last dim")
    if k_pool.shape != v_pool.shape or k_pool.dim() != 4 or not (k_pool.is_contiguous() and v_pool.is_contiguous()):
        raise ValueError("paged_decode_attention: pools must be contiguous [num_blocks, block_size, H_KV, D]")
    E, H, D = q.shape
    nb, bs, H_kv, Dk = k_pool.shape
    if Dk != D:
        raise ValueError(f"paged_decode_attention: head_dim {D} != pool head_dim {Dk}")
    if block_table.dtype != torch.int32 or context_len.dtype != torch.int32 or block_table.dim() != 2 \
            or block_table.stride(1) != 1 or context_len.shape != (E,) or block_table.shape[0] != E:
        raise ValueError("paged_decode_attention: block_table int32 [E, n] and context_len int32 [E]")
    if out is None:
        out = torch.empty((E, H, D), dtype=q.dtype, device=q.device)
    elif out.dtype != q.dtype or out.shape != (E, H, D) or out.stride(-1) != 1:
        raise ValueError("paged_decode_attention: out must be [E, H, D] of q's dtype with a contiguous last dim")
    if E == 0:
        return out
    _ensure_device(q.device)
    lib = _lib.load()
    stream = torch.cuda.current_stream(q.device)
    need = int(lib.lse_paged_decode_attention_workspace(E, H, H_kv, D, max_context, bs)) if split else 0
    key = (q.device.index, stream.cuda_stream)
    ws = _attn_ws.get(key)
    if need and (ws is None or ws.numel() < need):
        with _ws_lock:
            ws = _attn_ws.get(key)
            if ws is None or ws.numel() < need:
                if torch.cuda.is_current_stream_capturing():
                    raise RuntimeError("paged_decode_attention: workspace must grow outside a CUDA graph capture; "
                                       "run one eager call with the same shapes on the capture stream first")
                if ws is not None:
                    _attn_ws_retired.append(ws)
                ws = torch.zeros(need, dtype=torch.uint8, device=q.device)
                _attn_ws[key] = ws
    scale = 1.0 / float(D) ** 0.5 if scale is None else float(scale)
    rc = lib.lse_paged_decode_attention_dt(
        q.data_ptr(), _DTYPE_CODES[q.dtype], E, H, D, q.stride(0), q.stride(1), k_pool.data_ptr(), v_pool.data_ptr(), nb, bs, H_kv,
        block_table.data_ptr(), block_table.stride(0), context_len.data_ptr(), int(max_context), scale,
        out.data_ptr(), out.stride(0), out.stride(1), ws.data_ptr() if need else None, need, stream.cuda_stream)
    _lib.check(rc, "lse_paged_decode_attention_dt")
    return out


def paged_attention(q: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor, block_table: torch.Tensor,
                    context_len: torch.Tensor, query_offset: torch.Tensor, q_start: torch.Tensor, q_len: torch.Tensor,
                    block_size: int, max_q_len: int, scale: float | None = None,
                    out: torch.Tensor | None = None) -> torch.Tensor:
    """The reference's `paged_attention_forward` (`kernels/flash_attention.py:287-332`) on the
    sm_100a kernel, same arguments and result: q (H, tokens, D) bf16 or fp16 with d contiguous;
    k_pool / v_pool (num_blocks, block_size, H_KV, D) contiguous, same dtype; block_table
    int32 [E, n]; context_len, query_offset, q_start, q_len int32 [E]; max_q_len >= every
    q_len.  Returns o like q (a new tensor unless `out` is given): entry e's rows
    q_start[e] .. + q_len[e] - 1 attend causally (position query_offset[e] + i) to the
    positions below context_len[e].  Rows of no entry are left unwritten."""
    tensors = (q, k_pool, v_pool, block_table, context_len, query_offset, q_start, q_len)
    if not all(t.is_cuda for t in tensors):
        raise RuntimeError("paged_attention runs on CUDA only (no CPU fallback)")
    if q.dtype not in (torch.bfloat16, torch.float16) or k_pool.dtype != q.dtype or v_pool.dtype != q.dtype:
        raise ValueError("paged_attention: q and the pools must share a dtype, bfloat16 or float16")
    if q.dim() != 3 or q.stride(-1) != 1:
        raise ValueError("paged_attention: q must be (H, tokens, D) with a contiguous last dim")
    if k_pool.shape != v_pool.shape or k_pool.dim() != 4 or not (k_pool.is_contiguous() and v_pool.is_contiguous()):
        raise ValueError("paged_attention: pools must be contiguous (num_blocks, block_size, H_KV, D)")
    H, T, D = q.shape
    nb, bs, H_kv, Dk = k_pool.shape
    if Dk != D or bs != block_size:
        raise ValueError(f"paged_attention: pool (block_size {bs}, head_dim {Dk}) != ({block_size}, {D})")
    E = q_len.shape[0]
    for name, t in (("context_len", context_len), ("query_offset", query_offset), ("q_start", q_start),
                    ("q_len", q_len)):
        if t.dtype != torch.int32 or t.shape != (E,) or not t.is_contiguous():
            raise ValueError(f"paged_attention: {name} must be int32 [{E}]")
    if block_table.dtype != torch.int32 or block_table.dim() != 2 or block_table.shape[0] != E or block_table.stride(1) != 1:
        raise ValueError("paged_attention: block_table must be int32 [E, n] with contiguous rows")
    if out is None:
        out = torch.empty_like(q)
    elif out.dtype != q.dtype or out.shape != q.shape or out.stride(-1) != 1:
        raise ValueError("paged_attention: out must match q's dtype and shape with a contiguous last dim")
    if E == 0 or T == 0:
        return out
    _ensure_device(q.device)
    stream = torch.cuda.current_stream(q.device)
    scale = 1.0 / float(D) ** 0.5 if scale is None else float(scale)
    dt = _lib.DT_BF16 if q.dtype == torch.bfloat16 else _lib.DT_F16
    rc = _lib.load().lse_paged_attention(
        q.data_ptr(), dt, H, D, q.stride(0), q.stride(1), k_pool.data_ptr(), v_pool.data_ptr(), nb, bs, H_kv,
        block_table.data_ptr(), block_table.stride(0), context_len.data_ptr(), query_offset.data_ptr(),
        q_start.data_ptr(), q_len.data_ptr(), E, int(max_q_len), scale, out.data_ptr(), out.stride(0), out.stride(1),
        stream.cuda_stream)
    _lib.check(rc, "lse_paged_attention")
    return out


def set_wait_limit(cycles: int, device: int | torch.device | None = None) -> None:
    """Wait limit of the tensor-core kernels' data waits in SM cycles (lse_set_wait_limit);
    cycles <= 0 restores the default (~2 s).  For tests of the timeout path."""
    idx = _device_index(device)
    _lib.check(_lib.load().lse_set_wait_limit(idx, int(cycles)), "lse_set_wait_limit")


def _device_index(device: int | torch.device | None) -> int:
    if device is None:
        return torch.cuda.current_device()
    if isinstance(device, torch.device):
        return device.index if device.index is not None else torch.cuda.current_device()
    return int(device)


def device_status(device: int | torch.device | None = None, reset: bool = True) -> int:
    """Synchronize and read the device-side status (LSE_OK or LSE_ERR_DEVICE_TIMEOUT).  After a
    timeout the decode-attention workspaces of that device are re-zeroed (the linear
    workspaces need nothing: each call initialises its own)."""
    idx = _device_index(device)
    st = int(_lib.load().lse_device_status(idx, 1 if reset else 0))
    if st == _lib.LSE_ERR_DEVICE_TIMEOUT:
        for (d, _), ws in _attn_ws.items():
            if d == idx:
                ws.zero_()
    return st
