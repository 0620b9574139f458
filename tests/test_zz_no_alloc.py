"""lse_int8_linear_packed_noalloc: the tensor-core path with its scratch in the library's
fixed static device array instead of a caller workspace.

The file name sorts last, so in a full run these tests come after every other test (the
library's device state already set up by them); run alone, they start from a fresh process
in which the no-alloc call is the library's first.  Each GPU case calls the new entry point
twice in a row on one stream and checks both outputs against the existing entry point
(lse_int8_linear_packed with a caller workspace, LSE_ALGO_TCGEN05) on the same inputs,
within the parity tolerance of the other tests.
"""

from __future__ import annotations

import os
import re

import numpy as np
import pytest
import torch

from llm_serving_engine_b200 import _lib, ops
from llm_serving_engine_b200.inputs import make_inputs
from oracle.ref_linear import parity_errors
from tests.gpu_helpers import Workspace, check_parity, oracle_rows

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _noalloc(x: torch.Tensor, packed: torch.Tensor, s: torch.Tensor, N: int, K: int, y: torch.Tensor) -> int:
    return _lib.load().lse_int8_linear_packed_noalloc(
        x.data_ptr(), x.shape[0], K, x.stride(0), packed.data_ptr(), s.data_ptr(), N, y.data_ptr(), y.stride(0),
        torch.cuda.current_stream().cuda_stream)


def _existing(x, packed, s, N, K, ws: Workspace) -> torch.Tensor:
    ws.ensure(x.shape[0], K, N)
    y = torch.empty((x.shape[0], N), dtype=torch.bfloat16, device=x.device)
    rc = _lib.load().lse_int8_linear_packed(x.data_ptr(), x.shape[0], K, x.stride(0), packed.data_ptr(), s.data_ptr(),
                                            N, y.data_ptr(), y.stride(0), ws.ptr, ws.nbytes, _lib.ALGO_TCGEN05,
                                            torch.cuda.current_stream().cuda_stream)
    _lib.check(rc, "lse_int8_linear_packed")
    return y


def _nan_filled(M, N):
    return torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")


def _close(y: torch.Tensor, y_ref: torch.Tensor, what: str) -> None:
    a = y.float().cpu().numpy()
    b = y_ref.float().cpu().numpy().astype(np.float64)
    assert np.all(np.isfinite(a)), f"{what}: non-finite output"
    nw, ok, ratio = parity_errors(a, b)
    assert nw <= 1e-2, f"{what}: normwise difference {nw:.3e} > 1e-2"
    assert ok, f"{what}: elementwise criterion violated (worst ratio {ratio:.3f})"


def test_header_limits_match_binding():
    text = open(os.path.join(REPO, "include", "lse_int8.h")).read()
    assert int(re.search(r"#define LSE_NOALLOC_SCRATCH_BYTES (\d+)", text).group(1)) == _lib.NOALLOC_SCRATCH_BYTES
    assert int(re.search(r"#define LSE_NOALLOC_MAX_M (\d+)", text).group(1)) == _lib.NOALLOC_MAX_M


def test_rejects_m_beyond_limit_before_any_launch():
    """M > LSE_NOALLOC_MAX_M is refused on the host, before any CUDA call (runs on CPU)."""
    lib = _lib.load()
    rc = lib.lse_int8_linear_packed_noalloc(16, _lib.NOALLOC_MAX_M + 1, 64, 64, 16, 16, 32, 16, 32, None)
    assert rc == _lib.LSE_ERR_WORKSPACE
    msg = _lib.last_cuda_error()
    assert "LSE_NOALLOC_MAX_M" in msg and str(_lib.NOALLOC_MAX_M + 1) in msg
    assert lib.lse_int8_linear_packed_noalloc(16, -1, 64, 64, 16, 16, 32, 16, 32, None) == _lib.LSE_ERR_INVALID_ARG
    assert lib.lse_int8_linear_packed_noalloc(0, 0, 64, 64, 0, 0, 32, 0, 32, None) == _lib.LSE_OK


# (M, K, N): all of them run the 64-token tile (every M up to the limit does); the cases
# cover the schedules of the stream-K plan: a tile-aligned split (few tiles), data-parallel
# waves plus a stream-K tail (gate_up), an even spread with tiles shared between CTAs, and
# ragged N, M and K.
CASES = [(1, 256, 384), (17, 1024, 1536), (33, 4096, 1000), (64, 4096, 6144), (64, 4096, 28672), (48, 14336, 4096)]


@pytest.mark.gpu
@pytest.mark.parametrize("M,K,N", CASES)
def test_two_calls_in_a_row_match_workspace_path(M, K, N):
    x1, w, s = make_inputs(M, K, N, seed=11)
    x2 = make_inputs(M, K, N, seed=12)[0]
    xd1, xd2, sd = x1.cuda(), x2.cuda(), s.cuda()
    packed = ops.pack_weight(w.cuda())
    ws = Workspace()
    ref1 = _existing(xd1, packed, sd, N, K, ws)
    ref2 = _existing(xd2, packed, sd, N, K, ws)
    torch.cuda.synchronize()

    y1, y2 = _nan_filled(M, N), _nan_filled(M, N)
    _lib.check(_noalloc(xd1, packed, sd, N, K, y1), "lse_int8_linear_packed_noalloc (1st)")
    _lib.check(_noalloc(xd2, packed, sd, N, K, y2), "lse_int8_linear_packed_noalloc (2nd)")
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    _close(y1, ref1, f"1st call M={M} K={K} N={N}")
    _close(y2, ref2, f"2nd call M={M} K={K} N={N}")
    rows = np.unique([0, M // 2, M - 1])
    check_parity(y2[torch.as_tensor(rows, device="cuda")], oracle_rows(x2, w, s, rows), f"oracle M={M} K={K} N={N}")


@pytest.mark.gpu
def test_calls_allocate_no_device_memory():
    """After the first call (set-up), further calls leave the device's free memory as it was."""
    M, K, N = 64, 4096, 6144
    x, w, s = make_inputs(M, K, N, seed=13)
    xd, sd = x.cuda(), s.cuda()
    packed = ops.pack_weight(w.cuda())
    y = _nan_filled(M, N)
    _lib.check(_noalloc(xd, packed, sd, N, K, y), "lse_int8_linear_packed_noalloc")
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for _ in range(2):
        _lib.check(_noalloc(xd, packed, sd, N, K, y), "lse_int8_linear_packed_noalloc")
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0
    assert ops.device_status() == 0
