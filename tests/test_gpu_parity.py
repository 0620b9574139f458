"""Parity of the sm_100a kernels with the CPU oracle, called through the C ABI.

Tolerance (from the north_star): normwise max|y - ref| / max|ref| <= 1e-2 against the fp64
dequant-matmul oracle, and elementwise |y - ref| <= 1e-2*|ref| + 1e-3*max|ref|; bf16 output
rounding alone is ~2e-3 relative.  Full-size shapes are checked on a sample of rows of the
output (the oracle cost), plus size-independent properties (determinism, linearity in x,
zero inputs, workspace counters re-armed).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from llm_serving_engine_b200 import _lib, ops
from llm_serving_engine_b200.inputs import LLAMA3_8B_SHAPES, LLAMA3_70B_SHAPES, make_inputs
from oracle.ref_linear import ref_int8_linear, ref_quantize
from tests.gpu_helpers import Workspace, abi_linear, check_parity, oracle_rows

pytestmark = pytest.mark.gpu

ALGOS = {"gemv": _lib.ALGO_GEMV, "tcgen05": _lib.ALGO_TCGEN05, "auto": _lib.ALGO_AUTO, "skinny": _lib.ALGO_SKINNY}


@pytest.fixture(scope="module")
def ws():
    return Workspace()


def _run_case(M, K, N, algo, ws, seed=0, sample=None):
    x, w, s = make_inputs(M, K, N, seed=seed)
    xd, wd, sd = x.cuda(), w.cuda(), s.cuda()
    y = abi_linear(xd, wd, sd, ws, algo=algo)
    torch.cuda.synchronize()
    rows = np.arange(M) if sample is None or M <= sample else np.unique(
        np.concatenate([[0, M - 1], np.random.default_rng(seed).choice(M, sample, replace=False)]))
    ref = oracle_rows(x, w, s, rows)
    return check_parity(y[torch.as_tensor(rows, device="cuda")], ref, f"M={M} K={K} N={N} algo={algo}")


def test_config1_all_algos(ws):
    for name in ("gemv", "tcgen05", "auto"):
        _run_case(8, 2048, 2048, ALGOS[name], ws)
    assert ws.counters_clear() and ws.guard_intact()


@pytest.mark.parametrize("shape", list(LLAMA3_8B_SHAPES))
@pytest.mark.parametrize("M", [1, 4, 16, 64])
def test_decode_sweep_tcgen05(ws, shape, M):
    K, N = LLAMA3_8B_SHAPES[shape]
    _run_case(M, K, N, _lib.ALGO_TCGEN05, ws)
    assert ws.counters_clear() and ws.guard_intact()


@pytest.mark.parametrize("shape", list(LLAMA3_8B_SHAPES))
@pytest.mark.parametrize("M", [1, 2, 4])
def test_decode_sweep_gemv(ws, shape, M):
    K, N = LLAMA3_8B_SHAPES[shape]
    _run_case(M, K, N, _lib.ALGO_GEMV, ws)


@pytest.mark.parametrize("shape", list(LLAMA3_8B_SHAPES))
@pytest.mark.parametrize("M", [512, 2048])
def test_prefill_tcgen05(ws, shape, M):
    K, N = LLAMA3_8B_SHAPES[shape]
    _run_case(M, K, N, _lib.ALGO_TCGEN05, ws, sample=24)
    assert ws.counters_clear() and ws.guard_intact()


def _sample_rows(M: int, sample: int, seed: int) -> np.ndarray:
    if M <= sample:
        return np.arange(M)
    return np.unique(np.concatenate([[0, M - 1], np.random.default_rng(seed).choice(M, sample, replace=False)]))


@pytest.mark.parametrize("shape", list(LLAMA3_8B_SHAPES))
@pytest.mark.parametrize("M", [512, 2048, 8192])
def test_prefill_packed_auto_config3(ws, shape, M):
    """Config 3 as the modules and the bench run it: packed weights, automatic kernel choice,
    M up to 8192 (sampled rows against the oracle)."""
    K, N = LLAMA3_8B_SHAPES[shape]
    x, w, s = make_inputs(M, K, N, seed=M + N)
    packed = ops.pack_weight(w.cuda())
    y = _packed_call(x.cuda(), packed, s.cuda(), N, K, ws, _lib.ALGO_AUTO)
    torch.cuda.synchronize()
    rows = _sample_rows(M, 16, M + K)
    check_parity(y[torch.as_tensor(rows, device="cuda")], oracle_rows(x, w, s, rows), f"config3 {shape} M={M}")
    assert ws.counters_clear() and ws.guard_intact()


@pytest.fixture(scope="module", params=list(LLAMA3_70B_SHAPES))
def w70b(request):
    """One Llama-3-70B projection at full size: (name, K, N, W int8 [N, K] on the CPU, s, packed W on the GPU)."""
    K, N = LLAMA3_70B_SHAPES[request.param]
    g = torch.Generator().manual_seed(K + N)
    w = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int8)
    s = torch.empty(N).uniform_(1e-4, 5e-4, generator=g)
    packed = ops.pack_weight(w.cuda())
    yield request.param, K, N, w, s, packed
    del packed
    torch.cuda.empty_cache()


@pytest.mark.parametrize("M", [1, 32, 256, 4096])
def test_config5_70b_full_shapes_packed(ws, w70b, M):
    """Config 5's four 70B shapes at full size on the packed, automatic path (the one the module
    and the column split run), at the sweep's M values; sampled rows against the oracle."""
    name, K, N, w, s, packed = w70b
    x = torch.randn(M, K, generator=torch.Generator().manual_seed(M + 1)).to(torch.bfloat16)
    y = _packed_call(x.cuda(), packed, s.cuda(), N, K, ws, _lib.ALGO_AUTO)
    torch.cuda.synchronize()
    rows = _sample_rows(M, 6, M + N)
    check_parity(y[torch.as_tensor(rows, device="cuda")], oracle_rows(x, w, s, rows), f"config5 {name} M={M}")
    assert ws.counters_clear() and ws.guard_intact()


@pytest.mark.parametrize("M,K,N", [
    (1, 16, 8), (3, 48, 17), (17, 144, 136), (65, 4112, 200), (129, 272, 40), (7, 32, 64),
    (200, 64, 32), (16, 128, 128), (33, 256, 300), (1, 14336, 1000),
])
@pytest.mark.parametrize("algo", ["gemv", "tcgen05"])
def test_ragged_shapes(ws, M, K, N, algo):
    """Tails in every dimension: N and M not multiples of the tiles, K not a multiple of
    the 128-wide stage (TMA zero fill), tiny K, M past one token tile."""
    _run_case(M, K, N, ALGOS[algo], ws, seed=M + K + N)
    assert ws.counters_clear() and ws.guard_intact()


@pytest.mark.parametrize("algo", ["gemv", "tcgen05"])
def test_strided_x_and_y(ws, algo):
    M, K, N = 20, 256, 192
    x, w, s = make_inputs(M, K, N, seed=3)
    big = torch.zeros(M, K + 64, dtype=torch.bfloat16, device="cuda")
    big[:, :K] = x.cuda()
    ybig = torch.full((M, N + 24), 7.0, dtype=torch.bfloat16, device="cuda")
    abi_linear(big, w.cuda(), s.cuda(), ws, algo=ALGOS[algo], ldx=K + 64, y=ybig)
    torch.cuda.synchronize()
    check_parity(ybig[:, :N], oracle_rows(x, w, s, np.arange(M)), "strided")
    assert torch.all(ybig[:, N:] == 7.0), "wrote outside [M, N]"


@pytest.mark.parametrize("M", [1, 16, 64, 512])
def test_deterministic(ws, M):
    K, N = 4096, 4096
    x, w, s = make_inputs(M, K, N, seed=5)
    xd, wd, sd = x.cuda(), w.cuda(), s.cuda()
    a = abi_linear(xd, wd, sd, ws, algo=_lib.ALGO_TCGEN05)
    b = abi_linear(xd, wd, sd, ws, algo=_lib.ALGO_TCGEN05)
    torch.cuda.synchronize()
    assert torch.equal(a, b)


def test_linearity_full_size(ws):
    """y(2x) == 2 y(x) exactly (power-of-two scaling commutes with every rounding), at a
    full 8B gate_up shape where the oracle would be slow."""
    K, N = LLAMA3_8B_SHAPES["gate_up"]
    x, w, s = make_inputs(64, K, N, seed=9)
    xd, wd, sd = x.cuda(), w.cuda(), s.cuda()
    for algo in (_lib.ALGO_TCGEN05, _lib.ALGO_GEMV):
        y1 = abi_linear(xd[:4] if algo == _lib.ALGO_GEMV else xd, wd, sd, ws, algo=algo)
        y2 = abi_linear((xd[:4] if algo == _lib.ALGO_GEMV else xd) * 2, wd, sd, ws, algo=algo)
        torch.cuda.synchronize()
        assert torch.equal(y2, y1 * 2)


def test_zero_inputs(ws):
    K, N = 512, 256
    w = torch.randint(-127, 128, (N, K), dtype=torch.int8, device="cuda")
    s = torch.rand(N, device="cuda") + 0.1
    for algo in (_lib.ALGO_GEMV, _lib.ALGO_TCGEN05):
        y = abi_linear(torch.zeros(9, K, dtype=torch.bfloat16, device="cuda"), w, s, ws, algo=algo)
        torch.cuda.synchronize()
        assert torch.count_nonzero(y) == 0


def test_extreme_weights(ws):
    """All +-127 weights with the largest scale: no int overflow / saturation anywhere."""
    K, N = 14336, 256
    w = torch.full((N, K), 127, dtype=torch.int8)
    w[1::2] = -127
    s = torch.full((N,), 5e-4)
    x = torch.ones(16, K, dtype=torch.bfloat16)
    for algo in (_lib.ALGO_GEMV, _lib.ALGO_TCGEN05):
        y = abi_linear(x.cuda(), w.cuda(), s.cuda(), ws, algo=algo)
        torch.cuda.synchronize()
        check_parity(y, ref_int8_linear(x.float().numpy(), w.numpy(), s.numpy()), "extremes")


def test_quantize_kernel_bit_exact():
    g = torch.Generator().manual_seed(11)
    for dtype in (torch.float32, torch.bfloat16, torch.float16):
        w = (torch.randn(300, 1000, generator=g) * torch.rand(300, 1, generator=g) * 3).to(dtype)
        w[5] = 0
        q, s = ops.quantize_per_channel(w.cuda())
        qr, sr = ref_quantize(w.float().numpy())
        assert np.array_equal(q.cpu().numpy(), qr), dtype
        assert np.array_equal(s.cpu().numpy().view(np.uint32), sr.view(np.uint32)), dtype


def test_ops_wrapper_leading_dims_and_errors():
    x, w, s = make_inputs(6, 256, 96, seed=2)
    xd = x.cuda().view(2, 3, 256)
    y = ops.int8_linear(xd, w.cuda(), s.cuda())
    assert y.shape == (2, 3, 96) and y.dtype == torch.bfloat16
    check_parity(y.view(6, 96), ref_int8_linear(x.float().numpy(), w.numpy(), s.numpy()), "ops")
    with pytest.raises(ValueError):
        ops.int8_linear(xd.float(), w.cuda(), s.cuda())
    with pytest.raises(ValueError):
        ops.int8_linear(xd, w.cuda()[:, :128], s.cuda())
    with pytest.raises(ValueError):
        ops.int8_linear(torch.zeros(2, 24, dtype=torch.bfloat16, device="cuda"),
                        torch.zeros(8, 24, dtype=torch.int8, device="cuda"), torch.ones(8, device="cuda"))
    assert ops.int8_linear(torch.zeros(0, 256, dtype=torch.bfloat16, device="cuda"), w.cuda(), s.cuda()).shape == (0, 96)


def test_device_status_clean():
    assert ops.device_status() == _lib.LSE_OK


# ---- packed (tile-contiguous) weight layout ----------------------------------------------

@pytest.mark.parametrize("N,K", [(8, 16), (200, 272), (4096, 4096), (300, 14336)])
def test_pack_kernel_matches_layout_restatement(N, K):
    from oracle.ref_linear import ref_pack_weight

    w = torch.randint(-127, 128, (N, K), dtype=torch.int8, generator=torch.Generator().manual_seed(N + K))
    packed = ops.pack_weight(w.cuda())
    assert np.array_equal(packed.cpu().numpy(), ref_pack_weight(w.numpy()))
    assert torch.equal(ops.unpack_weight(packed, N, K).cpu(), w)


def _packed_call(x, packed, s, N, K, ws, algo, y=None, ldy=None):
    M = x.shape[0]
    ws.ensure(M, K, N)
    y = torch.empty(M, N, dtype=torch.bfloat16, device="cuda") if y is None else y
    ldy = y.stride(0) if ldy is None else ldy
    rc = _lib.load().lse_int8_linear_packed(x.data_ptr(), M, K, x.stride(0), packed.data_ptr(), s.data_ptr(), N,
                                            y.data_ptr(), ldy, ws.ptr, ws.nbytes, algo,
                                            torch.cuda.current_stream().cuda_stream)
    _lib.check(rc, "lse_int8_linear_packed")
    return y


@pytest.mark.parametrize("M,K,N", [(1, 16, 8), (3, 48, 17), (4, 4096, 6144), (9, 272, 200), (16, 144, 136),
                                   (2, 4096, 28672), (16, 4096, 28672), (5, 8192, 1040), (12, 8208, 272),
                                   (24, 4096, 4096), (31, 1040, 528),
                                   (17, 14336, 4096), (32, 4096, 28672), (64, 14336, 4096), (65, 4112, 200),
                                   (130, 1024, 640), (512, 4096, 4096)])
@pytest.mark.parametrize("algo", ["skinny", "tcgen05", "auto"])
def test_packed_path_parity(ws, M, K, N, algo):
    if algo == "skinny" and M > 32:
        pytest.skip("the skinny decode kernel serves M <= 32")
    x, w, s = make_inputs(M, K, N, seed=M * 7 + K + N)
    packed = ops.pack_weight(w.cuda())
    xd, sd = x.cuda(), s.cuda()
    y = _packed_call(xd, packed, sd, N, K, ws, ALGOS[algo])
    torch.cuda.synchronize()
    rows = np.arange(M) if M <= 64 else np.array([0, 1, M // 2, M - 1])
    check_parity(y[torch.as_tensor(rows, device="cuda")], oracle_rows(x, w, s, rows), f"packed {algo} M={M} K={K} N={N}")
    if algo == "tcgen05":
        # packed and row-major tensor-core paths run the same arithmetic in the same order
        y_rm = abi_linear(xd, w.cuda(), sd, ws, algo=_lib.ALGO_TCGEN05)
        torch.cuda.synchronize()
        assert torch.equal(y, y_rm)
    assert ws.counters_clear() and ws.guard_intact()


def test_packed_strided_and_layout_errors(ws):
    M, K, N = 12, 256, 192
    x, w, s = make_inputs(M, K, N, seed=4)
    packed = ops.pack_weight(w.cuda())
    big = torch.zeros(M, K + 64, dtype=torch.bfloat16, device="cuda")
    big[:, :K] = x.cuda()
    for algo in ("skinny", "tcgen05"):
        ybig = torch.full((M, N + 24), 7.0, dtype=torch.bfloat16, device="cuda")
        _packed_call(big, packed, s.cuda(), N, K, ws, ALGOS[algo], y=ybig)
        torch.cuda.synchronize()
        check_parity(ybig[:, :N], oracle_rows(x, w, s, np.arange(M)), f"packed strided {algo}")
        assert torch.all(ybig[:, N:] == 7.0)
    lib = _lib.load()
    y = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    assert lib.lse_int8_linear_packed(x.cuda().data_ptr(), M, K, K, packed.data_ptr(), s.cuda().data_ptr(), N,
                                      y.data_ptr(), N, ws.ptr, ws.nbytes, _lib.ALGO_GEMV, st) == _lib.LSE_ERR_UNSUPPORTED
    x40 = torch.zeros(40, K, dtype=torch.bfloat16, device="cuda")
    y40 = torch.empty(40, N, dtype=torch.bfloat16, device="cuda")
    assert lib.lse_int8_linear_packed(x40.data_ptr(), 40, K, K, packed.data_ptr(), s.cuda().data_ptr(), N,
                                      y40.data_ptr(), N, ws.ptr, ws.nbytes, _lib.ALGO_SKINNY, st) == _lib.LSE_ERR_UNSUPPORTED


@pytest.mark.parametrize("K,N", [(14336, 4096), (4096, 28672)])
@pytest.mark.parametrize("M", [1, 8, 9, 16, 17, 32])
def test_skinny_deterministic_and_linear(ws, M, K, N):
    x, w, s = make_inputs(M, K, N, seed=21)
    packed = ops.pack_weight(w.cuda())
    xd, sd = x.cuda(), s.cuda()
    a = _packed_call(xd, packed, sd, N, K, ws, _lib.ALGO_SKINNY)
    b = _packed_call(xd, packed, sd, N, K, ws, _lib.ALGO_SKINNY)
    c = _packed_call(xd * 2, packed, sd, N, K, ws, _lib.ALGO_SKINNY)
    torch.cuda.synchronize()
    assert torch.equal(a, b) and torch.equal(c, a * 2)


@pytest.mark.parametrize("M", [17, 24, 32])
@pytest.mark.parametrize("K,N,expect", [(4096, 6144, "skinny"), (4096, 4096, "skinny"), (8192, 4096, "skinny"),
                                        (14336, 4096, "tcgen05"), (4096, 8200, "tcgen05")])
def test_auto_choice_17_to_32_tokens(ws, M, K, N, expect):
    """From 17 to 32 tokens the automatic choice takes the decode kernel for weights of at most
    32 MiB (N * K) and the tensor-core kernel above: bit for bit the pinned algorithm's result,
    within the parity criterion of the oracle either way."""
    x, w, s = make_inputs(M, K, N, seed=M + N)
    packed = ops.pack_weight(w.cuda())
    xd, sd = x.cuda(), s.cuda()
    auto = _packed_call(xd, packed, sd, N, K, ws, _lib.ALGO_AUTO)
    pinned = _packed_call(xd, packed, sd, N, K, ws, ALGOS[expect])
    torch.cuda.synchronize()
    assert torch.equal(auto, pinned), f"M={M} K={K} N={N}: auto is not {expect}"
    rows = np.unique(np.linspace(0, M - 1, 6).astype(int))
    check_parity(auto[torch.as_tensor(rows, device="cuda")], oracle_rows(x, w, s, rows), f"auto M={M} K={K} N={N}")
    assert ws.counters_clear() and ws.guard_intact()


@pytest.mark.parametrize("M,K,N", [(64, 4096, 28672), (40, 1040, 33240), (33, 2048, 30720)])
def test_whole_tiles_over_one_and_a_half_waves(ws, M, K, N):
    """64-token tiles over more than one wave with the last wave at least half full run whole
    tiles round-robin (224, 260 and 240 tiles: some CTAs take two, ragged N and K included):
    parity with the oracle on sampled rows and columns, deterministic, linear in x, and no
    stream-K counter left set."""
    x, w, s = make_inputs(M, K, N, seed=N + M)
    packed = ops.pack_weight(w.cuda())
    xd, sd = x.cuda(), s.cuda()
    a = _packed_call(xd, packed, sd, N, K, ws, _lib.ALGO_TCGEN05)
    b = _packed_call(xd, packed, sd, N, K, ws, _lib.ALGO_TCGEN05)
    c = _packed_call(xd * 2, packed, sd, N, K, ws, _lib.ALGO_TCGEN05)
    torch.cuda.synchronize()
    assert torch.equal(a, b) and torch.equal(c, a * 2)
    rows = np.unique(np.linspace(0, M - 1, 5).astype(int))
    cols = np.unique(np.concatenate([np.arange(0, N, 97), [N - 1]]))
    ref = oracle_rows(x, w[cols], s[cols], rows)
    got = a[torch.as_tensor(rows, device="cuda")][:, torch.as_tensor(cols, device="cuda")]
    check_parity(got, ref, f"whole tiles M={M} K={K} N={N}")
    assert ws.counters_clear() and ws.guard_intact()


# ---- fused gate_up + SiLU * mul (decode) ------------------------------------------------
def _silu_mul_ref(x, qg, sg, qu, su):
    g = ref_int8_linear(x, qg, sg)
    u = ref_int8_linear(x, qu, su)
    return (g / (1.0 + np.exp(-g))) * u


@pytest.mark.parametrize("M,K,I", [(1, 256, 512), (3, 512, 200), (5, 272, 496), (8, 4096, 2048), (9, 1024, 1024),
                                   (13, 208, 1032), (16, 4096, 14336)])
def test_gate_up_silu_fused_parity(M, K, I):
    g = torch.Generator().manual_seed(M + K + I)
    x = (torch.randn(M, K, generator=g) * 0.5).to(torch.bfloat16)
    qg = torch.randint(-127, 128, (I, K), generator=g, dtype=torch.int8)
    qu = torch.randint(-127, 128, (I, K), generator=g, dtype=torch.int8)
    sg = torch.empty(I).uniform_(1e-4, 5e-4, generator=g)
    su = torch.empty(I).uniform_(1e-4, 5e-4, generator=g)
    perm = ops.interleave_gate_up_rows(I)
    q = torch.cat([qg, qu]).index_select(0, perm)
    s = torch.cat([sg, su]).index_select(0, perm)
    packed = ops.pack_weight(q.cuda())
    y = ops.int8_gate_up_silu_packed(x.cuda(), packed, s.cuda(), I, K)
    torch.cuda.synchronize()
    cols = np.arange(I) if I <= 2048 else np.unique(np.random.default_rng(0).choice(I, 2048, replace=False))
    ref = _silu_mul_ref(x.float().numpy(), qg.numpy()[cols], sg.numpy()[cols], qu.numpy()[cols], su.numpy()[cols])
    check_parity(y[:, torch.as_tensor(cols, device="cuda")], ref, f"gate_up silu M={M} K={K} I={I}")
    assert ops.device_status() == 0


def test_gate_up_silu_fused_limits():
    lib = _lib.load()
    st = torch.cuda.current_stream().cuda_stream
    x = torch.zeros(17, 64, dtype=torch.bfloat16, device="cuda")
    w = torch.zeros(ops.packed_weight_bytes(64, 64), dtype=torch.int8, device="cuda")
    s = torch.ones(64, device="cuda")
    y = torch.empty(17, 32, dtype=torch.bfloat16, device="cuda")
    assert lib.lse_int8_gate_up_silu_packed(x.data_ptr(), 17, 64, 64, w.data_ptr(), s.data_ptr(), 32, y.data_ptr(), 32,
                                            st) == _lib.LSE_ERR_UNSUPPORTED
    assert lib.lse_int8_gate_up_silu_packed(x.data_ptr(), 4, 64, 64, w.data_ptr(), s.data_ptr(), 20, y.data_ptr(), 32,
                                            st) == _lib.LSE_ERR_UNSUPPORTED  # I % 8
    # K == 0: silu(0) * 0 = 0
    y.fill_(1.0)
    assert lib.lse_int8_gate_up_silu_packed(x.data_ptr(), 4, 0, 64, w.data_ptr(), s.data_ptr(), 32, y.data_ptr(), 32,
                                            st) == _lib.LSE_OK
    torch.cuda.synchronize()
    assert torch.all(y[:4] == 0)


# ---- the same fused on the tensor-core path (M > 16, SiLU * mul in the tcgen05 epilogue) ----
@pytest.mark.parametrize("M,K,I", [(17, 256, 512), (40, 512, 200), (64, 4096, 14336), (65, 272, 1032),
                                   (200, 1024, 1024), (512, 4096, 14336), (2048, 512, 2048)])
def test_gate_up_silu_fused_tc_parity(M, K, I):
    """Whole tiles (M = 2048: 296 data-parallel tiles), stream-K tiles finished by the last
    arriving CTA (M = 64: every tile), ragged rows (I = 200, 1032) and ragged tokens."""
    g = torch.Generator().manual_seed(M + K + I)
    x = (torch.randn(M, K, generator=g) * 0.5).to(torch.bfloat16)
    qg = torch.randint(-127, 128, (I, K), generator=g, dtype=torch.int8)
    qu = torch.randint(-127, 128, (I, K), generator=g, dtype=torch.int8)
    sg = torch.empty(I).uniform_(1e-4, 5e-4, generator=g)
    su = torch.empty(I).uniform_(1e-4, 5e-4, generator=g)
    perm = ops.interleave_gate_up_rows(I)
    q = torch.cat([qg, qu]).index_select(0, perm)
    s = torch.cat([sg, su]).index_select(0, perm)
    packed = ops.pack_weight(q.cuda())
    xd = x.cuda()
    y = ops.int8_gate_up_silu_packed(xd, packed, s.cuda(), I, K)
    y2 = ops.int8_gate_up_silu_packed(xd, packed, s.cuda(), I, K)
    torch.cuda.synchronize()
    assert torch.equal(y, y2)  # fixed reduction order
    rows = np.arange(M) if M <= 256 else np.unique(np.random.default_rng(1).choice(M, 256, replace=False))
    cols = np.arange(I) if I <= 2048 else np.unique(np.random.default_rng(0).choice(I, 2048, replace=False))
    ref = _silu_mul_ref(x.float().numpy()[rows], qg.numpy()[cols], sg.numpy()[cols], qu.numpy()[cols], su.numpy()[cols])
    got = y[torch.as_tensor(rows, device="cuda")][:, torch.as_tensor(cols, device="cuda")]
    check_parity(got, ref, f"gate_up silu (tcgen05) M={M} K={K} I={I}")
    # the unfused path on the same weights: projection, then SiLU * mul of the paired rows
    gu = ops.int8_linear_packed(xd, packed, s.cuda(), 2 * I, K).view(M, I // 8, 2, 8).float()
    unf = (torch.nn.functional.silu(gu[:, :, 0]) * gu[:, :, 1]).reshape(M, I)
    assert (y.float() - unf).abs().max().item() <= 2e-2 * unf.abs().max().item()
    assert ops.device_status() == 0


def test_gate_up_silu_ws_limits():
    lib = _lib.load()
    st = torch.cuda.current_stream().cuda_stream
    x = torch.zeros(40, 64, dtype=torch.bfloat16, device="cuda")
    w = torch.zeros(ops.packed_weight_bytes(64, 64), dtype=torch.int8, device="cuda")
    s = torch.ones(64, device="cuda")
    y = torch.empty(40, 32, dtype=torch.bfloat16, device="cuda")
    ws = torch.empty(int(lib.lse_int8_linear_workspace(40, 64, 64)), dtype=torch.uint8, device="cuda")
    assert lib.lse_int8_gate_up_silu_packed_ws(x.data_ptr(), 40, 64, 64, w.data_ptr(), s.data_ptr(), 32, y.data_ptr(),
                                               32, None, 0, st) == _lib.LSE_ERR_WORKSPACE
    assert lib.lse_int8_gate_up_silu_packed_ws(x.data_ptr(), 40, 64, 64, w.data_ptr(), s.data_ptr(), 20, y.data_ptr(),
                                               32, ws.data_ptr(), ws.numel(), st) == _lib.LSE_ERR_UNSUPPORTED  # I % 8
    y.fill_(1.0)
    assert lib.lse_int8_gate_up_silu_packed_ws(x.data_ptr(), 40, 0, 64, w.data_ptr(), s.data_ptr(), 32, y.data_ptr(),
                                               32, ws.data_ptr(), ws.numel(), st) == _lib.LSE_OK
    torch.cuda.synchronize()
    assert torch.all(y == 0)  # K == 0: silu(0) * 0


@pytest.mark.parametrize("M", [4, 40])
def test_tensor_parallel_mlp_fused_path_one_rank(M):
    """TensorParallelInt8MLP without a process group (one rank): gate_up + SiLU * mul fused on
    the rank's 8-row interleaved rows, against the fp64 MLP oracle and against the unfused
    projections on the same weights (normwise: the two round the intermediate differently)."""
    import torch.nn.functional as F
    from llm_serving_engine_b200.int8_linear import Int8Linear
    from llm_serving_engine_b200.parallel import TensorParallelInt8MLP
    from oracle.ref_linear import ref_mlp
    H, I = 512, 1024
    g = torch.Generator().manual_seed(M)
    wg, wu, wd = (torch.randn(*shape, generator=g) * 0.02 for shape in [(I, H), (I, H), (H, I)])
    qs = [ops.quantize_per_channel(t.cuda()) for t in (wg, wu, wd)]
    x = torch.randn(M, H, generator=g).to(torch.bfloat16).cuda()
    mlp = TensorParallelInt8MLP.from_quantized(qs[0][0], qs[0][1], qs[1][0], qs[1][1], qs[2][0], qs[2][1])
    assert mlp.fused
    y = mlp(x).float().cpu().numpy()
    gu = Int8Linear.from_quantized(torch.cat([qs[0][0], qs[1][0]]), torch.cat([qs[0][1], qs[1][1]]))(x)
    unfused = Int8Linear.from_quantized(*qs[2])(F.silu(gu[:, :I]) * gu[:, I:]).float().cpu().numpy()
    q_np = [(q.cpu().numpy(), s.cpu().numpy()) for q, s in qs]
    ref = ref_mlp(x.float().cpu().numpy(), *q_np[0], *q_np[1], *q_np[2])
    # the bf16 rounding of the intermediate between the two projections adds ~1e-2
    assert np.max(np.abs(y - ref)) / np.max(np.abs(ref)) < 2e-2
    assert np.max(np.abs(y - unfused)) / np.max(np.abs(unfused)) < 1e-2
    assert ops.device_status() == 0


@pytest.mark.parametrize("M", [3, 16, 40])
def test_mlp_module_fused_and_unfused_paths(M):
    """Int8LlamaMLP runs gate_up + SiLU * mul fused for every M (the decode kernel up to 16
    tokens, the tensor-core kernel above), against the fp64 MLP oracle."""
    from llm_serving_engine_b200.int8_linear import Int8LlamaMLP
    from oracle.ref_linear import ref_mlp
    H, I = 512, 1024
    g = torch.Generator().manual_seed(M)
    qg, qu = (torch.randint(-127, 128, (I, H), generator=g, dtype=torch.int8) for _ in range(2))
    qd = torch.randint(-127, 128, (H, I), generator=g, dtype=torch.int8)
    sg, su = (torch.empty(I).uniform_(1e-4, 5e-4, generator=g) for _ in range(2))
    sd = torch.empty(H).uniform_(1e-4, 5e-4, generator=g)
    from llm_serving_engine_b200.int8_linear import Int8Linear
    mlp = Int8LlamaMLP(Int8Linear.from_quantized(torch.cat([qg, qu]).cuda(), torch.cat([sg, su]).cuda()),
                       Int8Linear.from_quantized(qd.cuda(), sd.cuda()), I)
    assert torch.equal(mlp.gate_weight().cpu(), (qg.float() * sg[:, None]))
    x = (torch.randn(M, H, generator=g) * 4).to(torch.bfloat16)
    y = mlp(x.cuda()).float().cpu().numpy()
    ref = ref_mlp(x.float().numpy(), qg.numpy(), sg.numpy(), qu.numpy(), su.numpy(), qd.numpy(), sd.numpy())
    # the bf16 rounding of the intermediate between the two projections adds ~1e-2
    assert np.max(np.abs(y - ref)) / np.max(np.abs(ref)) < 2e-2


# ---- residual add fused into the epilogue ------------------------------------------------
@pytest.mark.parametrize("M,K,N,algo", [
    (1, 4096, 1024, ops.ALGO_AUTO),      # skinny, fp16 MMA
    (5, 1040, 528, ops.ALGO_AUTO),       # skinny, ragged K and N
    (16, 2048, 2048, ops.ALGO_AUTO),     # skinny, bf16 MMA
    (24, 1024, 1024, ops.ALGO_SKINNY),   # skinny, four token tiles
    (64, 8192, 1024, ops.ALGO_AUTO),     # tensor cores, stream-K reductions
    (300, 2048, 2176, ops.ALGO_AUTO),    # tensor cores, 128-token tiles
])
def test_residual_epilogue_parity(M, K, N, algo):
    x, w, s = make_inputs(M, K, N, seed=M * 7 + N)
    g = torch.Generator().manual_seed(M + K)
    res = (torch.randn(M, N, generator=g) * 0.05).to(torch.bfloat16)
    wp = ops.pack_weight(w.cuda())
    y = ops.int8_linear_packed(x.cuda(), wp, s.cuda(), N, K, algo=algo, residual=res.cuda())
    torch.cuda.synchronize()
    ref = ref_int8_linear(x.float().numpy(), w.numpy(), s.numpy()) + res.double().numpy()
    check_parity(y, ref, f"residual M={M} K={K} N={N}")
    # in place: the residual stream is updated where it lies
    h = res.cuda().clone()
    out = ops.int8_linear_packed(x.cuda(), wp, s.cuda(), N, K, algo=algo, residual=h, out=h)
    torch.cuda.synchronize()
    assert out.data_ptr() == h.data_ptr()
    assert torch.equal(h, y)
    assert ops.device_status() == 0


def test_residual_argument_errors():
    lib = _lib.load()
    st = torch.cuda.current_stream().cuda_stream
    x = torch.zeros(4, 64, dtype=torch.bfloat16, device="cuda")
    wp = torch.zeros(ops.packed_weight_bytes(64, 64), dtype=torch.int8, device="cuda")
    s = torch.ones(64, device="cuda")
    y = torch.empty(4, 64, dtype=torch.bfloat16, device="cuda")
    ws = torch.empty(int(lib.lse_int8_linear_workspace(4, 64, 64)), dtype=torch.uint8, device="cuda")
    args = (x.data_ptr(), 4, 64, 64, wp.data_ptr(), s.data_ptr(), 64)
    tail = (ws.data_ptr(), ws.numel(), ops.ALGO_AUTO, st)
    assert lib.lse_int8_linear_packed_residual(*args, None, 64, y.data_ptr(), 64, *tail) == _lib.LSE_ERR_INVALID_ARG
    assert lib.lse_int8_linear_packed_residual(*args, y.data_ptr(), 32, y.data_ptr(), 64, *tail) == _lib.LSE_ERR_INVALID_ARG
    r = torch.empty(4, 128, dtype=torch.bfloat16, device="cuda")
    # same pointer as y with another row stride would overlap element for element differently
    assert lib.lse_int8_linear_packed_residual(*args, y.data_ptr(), 128, y.data_ptr(), 64, *tail) == _lib.LSE_ERR_INVALID_ARG
    # K == 0: y = residual
    r[:, :64] = 3.0
    assert lib.lse_int8_linear_packed_residual(x.data_ptr(), 4, 0, 64, wp.data_ptr(), s.data_ptr(), 64, r.data_ptr(), 128,
                                               y.data_ptr(), 64, *tail) == _lib.LSE_OK
    torch.cuda.synchronize()
    assert torch.all(y == 3.0)
    with pytest.raises(ValueError):
        ops.int8_linear_packed(x, wp, s, 64, 64, residual=torch.zeros(4, 32, dtype=torch.bfloat16, device="cuda"))
