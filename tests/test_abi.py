"""The C-ABI library builds, loads without a GPU, exports every declared symbol, and rejects
bad arguments on the host before any launch (CPU only)."""

from __future__ import annotations

import ctypes
import os
import re

import pytest

from llm_serving_engine_b200 import _lib, build

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "lse_int8.h")


def declared_functions() -> list[str]:
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(lse_[a-z0-9_]+)\s*\(", text)))


def test_library_builds_and_loads():
    path = build.build()
    assert os.path.exists(path)
    lib = _lib.load()
    assert lib.lse_abi_version() == _lib.ABI_VERSION


def test_every_declared_symbol_is_exported_and_bound():
    lib = _lib.load()
    names = declared_functions()
    assert "lse_int8_linear" in names and "lse_int8_quantize" in names
    for name in names:
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"


def test_header_constants_match_binding():
    text = open(HEADER).read()
    assert int(re.search(r"#define LSE_WS_COUNTER_BYTES (\d+)", text).group(1)) == _lib.WS_COUNTER_BYTES
    assert int(re.search(r"#define LSE_ABI_VERSION (\d+)", text).group(1)) == _lib.ABI_VERSION
    for name, val in [("LSE_ERR_ALIGNMENT", _lib.LSE_ERR_ALIGNMENT), ("LSE_ERR_WORKSPACE", _lib.LSE_ERR_WORKSPACE),
                      ("LSE_ERR_DEVICE_TIMEOUT", _lib.LSE_ERR_DEVICE_TIMEOUT)]:
        assert re.search(rf"{name} = {val}\b", text), name


def test_status_strings():
    for st in range(7):
        assert _lib.status_string(st)
    assert _lib.status_string(99) == "unknown status"


def _call(M=4, K=64, ldx=64, N=32, ldy=32, x=16, w=16, s=16, y=16, ws=16, wsb=1 << 26, algo=0):
    lib = _lib.load()
    return lib.lse_int8_linear_ex(x, M, K, ldx, w, s, N, y, ldy, ws, wsb, algo, None)


def test_host_validation_rejects_before_launch():
    # no device is touched for these: validation precedes every CUDA call
    assert _call(M=-1) == _lib.LSE_ERR_INVALID_ARG
    assert _call(M=0) == _lib.LSE_OK and _call(N=0) == _lib.LSE_OK
    assert _call(x=0) == _lib.LSE_ERR_INVALID_ARG
    assert _call(ldx=32) == _lib.LSE_ERR_INVALID_ARG
    assert _call(ldy=16) == _lib.LSE_ERR_INVALID_ARG
    assert _call(K=24, ldx=24) == _lib.LSE_ERR_ALIGNMENT
    assert _call(ldx=68) == _lib.LSE_ERR_ALIGNMENT
    assert _call(x=24) == _lib.LSE_ERR_ALIGNMENT
    assert _call(w=8) == _lib.LSE_ERR_ALIGNMENT
    assert _call(algo=7) == _lib.LSE_ERR_INVALID_ARG
    assert _call(algo=_lib.ALGO_SKINNY) == _lib.LSE_ERR_UNSUPPORTED  # skinny needs packed W
    lib = _lib.load()
    assert lib.lse_int8_quantize(None, 0, 4, 4, 4, None, None, None) == _lib.LSE_ERR_INVALID_ARG
    assert lib.lse_int8_quantize(16, 0, 4, 8, 4, 16, 16, None) == _lib.LSE_ERR_INVALID_ARG


def test_workspace_size_covers_counter_region():
    lib = _lib.load()
    for M in (1, 16, 17, 64, 65, 8192):
        assert lib.lse_int8_linear_workspace(M, 4096, 4096) > _lib.WS_COUNTER_BYTES
    assert lib.lse_int8_linear_workspace(0, 1, 1) == _lib.WS_COUNTER_BYTES


def test_workspace_for_follows_the_kernel_choice():
    """No scratch where the decode kernel (packed, M <= 16, or M <= 32 with N * K <= 32 MiB)
    or the GEMV (row-major, M <= 2) runs; the tensor-core size everywhere else, growing with M
    and K (digit planes)."""
    lib = _lib.load()
    for M in (1, 8, 16):
        assert lib.lse_int8_linear_workspace_for(M, 4096, 4096, _lib.ALGO_AUTO, 1) == 0
        assert lib.lse_int8_linear_workspace_for(M, 4096, 4096, _lib.ALGO_SKINNY, 1) == 0
        assert lib.lse_int8_linear_workspace_for(M, 14336, 4096, _lib.ALGO_AUTO, 1) == 0
    for M in (17, 32):  # by the weight's size
        for K, N in ((4096, 6144), (4096, 8192), (8192, 4096)):
            assert lib.lse_int8_linear_workspace_for(M, K, N, _lib.ALGO_AUTO, 1) == 0
        for K, N in ((4096, 8200), (14336, 4096), (4096, 28672)):
            need = lib.lse_int8_linear_workspace_for(M, K, N, _lib.ALGO_AUTO, 1)
            assert need == lib.lse_int8_linear_workspace(M, K, N) > _lib.WS_COUNTER_BYTES
    for M in (1, 2):
        assert lib.lse_int8_linear_workspace_for(M, 4096, 4096, _lib.ALGO_AUTO, 0) == 0
    for M, packed in ((33, 1), (17, 0), (3, 0), (64, 1), (4096, 0)):
        need = lib.lse_int8_linear_workspace_for(M, 4096, 4096, _lib.ALGO_AUTO, packed)
        assert need == lib.lse_int8_linear_workspace(M, 4096, 4096) > _lib.WS_COUNTER_BYTES
    assert lib.lse_int8_linear_workspace_for(4, 4096, 4096, _lib.ALGO_TCGEN05, 1) > 0
    assert lib.lse_int8_linear_workspace(512, 8192, 64) > lib.lse_int8_linear_workspace(512, 4096, 64)
    assert lib.lse_int8_linear_workspace(1024, 4096, 64) > lib.lse_int8_linear_workspace(512, 4096, 64)


def test_no_cpu_fallback():
    import torch

    from llm_serving_engine_b200 import ops

    x = torch.zeros(2, 16, dtype=torch.bfloat16)
    w = torch.zeros(4, 16, dtype=torch.int8)
    s = torch.ones(4)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.int8_linear(x, w, s)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.quantize_per_channel(torch.zeros(4, 16))


def test_library_has_no_libcuda_link_dependency():
    """Loads on hosts without a driver: libcuda is reached only through the runtime's
    driver-entry-point query."""
    import subprocess

    deps = subprocess.run(["ldd", build.LIB_PATH], capture_output=True, text=True).stdout
    assert "libcuda.so" not in deps and "libcudart" not in deps, deps
    ctypes.CDLL(build.LIB_PATH)


def test_attention_rope_norm_host_validation():
    """The decode-attention, RoPE/K-V and RMSNorm entries refuse bad arguments on the host,
    before any device call (no GPU here)."""
    lib = _lib.load()
    P = 256  # any 256-aligned non-null address: never dereferenced on these paths
    # H not a multiple of H_kv; head_dim 96; block table narrower than max_context / block_size
    assert lib.lse_paged_decode_attention(P, 2, 12, 128, 1536, 128, P, P, 10, 16, 8, P, 4, P, 64, 0.1, P, 1536, 128,
                                          None, 0, None) == _lib.LSE_ERR_INVALID_ARG
    assert lib.lse_paged_decode_attention(P, 2, 8, 96, 768, 96, P, P, 10, 16, 8, P, 4, P, 64, 0.1, P, 768, 96,
                                          None, 0, None) == _lib.LSE_ERR_UNSUPPORTED
    assert lib.lse_paged_decode_attention(P, 2, 8, 128, 1024, 128, P, P, 10, 16, 8, P, 3, P, 64, 0.1, P, 1024, 128,
                                          None, 0, None) == _lib.LSE_ERR_INVALID_ARG
    assert lib.lse_paged_decode_attention(P + 1, 2, 8, 128, 1024, 128, P, P, 10, 16, 8, P, 4, P, 64, 0.1, P, 1024,
                                          128, None, 0, None) == _lib.LSE_ERR_ALIGNMENT
    assert lib.lse_paged_decode_attention(P, 0, 8, 128, 1024, 128, P, P, 10, 16, 8, P, 4, P, 64, 0.1, P, 1024, 128,
                                          None, 0, None) == _lib.LSE_OK  # no sequences: nothing to do
    # odd head_dim; cos/sin dtype code outside {F32, BF16, F16}; rows of another type
    assert lib.lse_rope_kv_write(P, 4, 1000, 8, 2, 63, P, P, 63, _lib.DT_F32, P, P, P, P, 63, None) == \
        _lib.LSE_ERR_INVALID_ARG
    assert lib.lse_rope_kv_write(P, 4, 1536, 8, 2, 128, P, P, 128, 7, P, P, P, P, 128, None) == \
        _lib.LSE_ERR_INVALID_ARG
    assert lib.lse_rope_kv_write_dt(P, _lib.DT_F32, 4, 1536, 8, 2, 128, P, P, 128, _lib.DT_F32, P, P, P, P, 128,
                                    None) == _lib.LSE_ERR_UNSUPPORTED
    assert lib.lse_rms_norm_dt(P, _lib.DT_F32, 4, 64, 64, P, 1e-5, P, 64, None) == _lib.LSE_ERR_UNSUPPORTED
    # RMSNorm: N % 8, ld < N, negative eps
    assert lib.lse_rms_norm(P, 4, 12, 16, P, 1e-5, P, 16, None) == _lib.LSE_ERR_ALIGNMENT
    assert lib.lse_rms_norm(P, 4, 64, 32, P, 1e-5, P, 64, None) == _lib.LSE_ERR_INVALID_ARG
    assert lib.lse_rms_norm(P, 4, 64, 64, P, -1.0, P, 64, None) == _lib.LSE_ERR_INVALID_ARG


def test_gate_up_silu_host_validation():
    """Both fused gate_up + SiLU*mul entries refuse bad arguments on the host (no GPU here)."""
    lib = _lib.load()
    P = 256
    for M in (4, 40):  # the decode-kernel entry's range, and the tensor-core range of the _ws entry
        ws = lib.lse_int8_gate_up_silu_packed_ws
        assert ws(P, M, 64, 64, P, P, 20, P, 32, P, 1 << 26, None) == _lib.LSE_ERR_UNSUPPORTED  # I % 8
        assert ws(P, M, 64, 64, P, P, 32, P, 16, P, 1 << 26, None) == _lib.LSE_ERR_INVALID_ARG  # ldy < I
        assert ws(P, M, 64, 32, P, P, 32, P, 32, P, 1 << 26, None) == _lib.LSE_ERR_INVALID_ARG  # ldx < K
        assert ws(P + 8, M, 64, 64, P, P, 32, P, 32, P, 1 << 26, None) == _lib.LSE_ERR_ALIGNMENT
        assert ws(P, M, 64, 64, P, P, 32, P + 1, 32, P, 1 << 26, None) == _lib.LSE_ERR_ALIGNMENT
        assert ws(None, M, 64, 64, P, P, 32, P, 32, P, 1 << 26, None) == _lib.LSE_ERR_INVALID_ARG
        assert ws(P, M, 64, 64, P, P, 0, P, 32, P, 1 << 26, None) == _lib.LSE_OK  # I == 0: nothing to do
    assert lib.lse_int8_gate_up_silu_packed_ws(P, -1, 64, 64, P, P, 32, P, 32, P, 1 << 26, None) == \
        _lib.LSE_ERR_INVALID_ARG
    # the decode-kernel entry alone stops at 16 tokens
    assert lib.lse_int8_gate_up_silu_packed(P, 17, 64, 64, P, P, 32, P, 32, None) == _lib.LSE_ERR_UNSUPPORTED


def test_python_ops_refuse_cpu_tensors():
    """No CPU fallback: the torch-facing ops raise on CPU tensors."""
    import torch

    from llm_serving_engine_b200 import ops

    q = torch.zeros(2, 8, 64, dtype=torch.bfloat16)
    pool = torch.zeros(4, 16, 2, 64, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA only"):
        ops.paged_decode_attention(q, pool, pool, torch.zeros(2, 2, dtype=torch.int32),
                                   torch.ones(2, dtype=torch.int32), 16)
    with pytest.raises(ValueError):
        ops.rms_norm(torch.zeros(2, 64), torch.ones(64), 1e-5)
    with pytest.raises((RuntimeError, ValueError)):
        ops.rope_kv_write(torch.zeros(2, 12 * 64, dtype=torch.bfloat16), 8, 2, 64, torch.zeros(2, 64),
                          torch.zeros(2, 64), pool, pool, torch.zeros(2, dtype=torch.int64))


def test_torch_operators_register_without_a_gpu():
    """liblse_torch.so loads on a machine without a GPU and registers the two operators with
    the documented schemas; they have no CPU kernel (a CPU call is refused, nothing falls back)."""
    import torch

    from llm_serving_engine_b200 import ops

    lse = ops.torch_ops()
    assert str(lse.int8_linear.default._schema) == (
        "lse::int8_linear(Tensor x, Tensor w_packed, Tensor scale, int N, int K, Tensor? residual=None, "
        "int algo=0) -> Tensor")
    assert str(lse.gate_up_silu.default._schema) == (
        "lse::gate_up_silu(Tensor x, Tensor w_packed, Tensor scale, int I, int K) -> Tensor")
    with pytest.raises((NotImplementedError, RuntimeError)):
        lse.int8_linear(torch.zeros(2, 16, dtype=torch.bfloat16), torch.zeros(2048, dtype=torch.int8),
                        torch.ones(16), 16, 16)
