"""RMSNorm fused with the projection that consumes it (`ops.rms_norm_proj`,
`lse_int8_rms_norm_linear_packed` / `lse_int8_rms_norm_gate_up_silu_packed`): bitwise the same
as `rms_norm` followed by the packed projection (the decode kernel up to 16 tokens, the
tensor-core kernel with the normalisation writing its digit planes above), and within the
parity criterion of the fp64 oracle of the reference's arithmetic (LlamaRMSNorm then
nn.Linear / LlamaMLP).  Covers the cluster and stream-K schedules, ragged K, a row longer than
the normalisation keeps in registers, and the refusals before any launch."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from llm_serving_engine_b200 import _lib, ops
from llm_serving_engine_b200.inputs import make_inputs
from tests.gpu_helpers import check_parity, oracle_rows

pytestmark = pytest.mark.gpu

EPS = 1e-5


def _norm_ref(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """The normalised rows as the kernels round them (bf16), for the oracle's input."""
    xf = x.float()
    r = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + EPS)
    return ((xf * r).to(torch.bfloat16).float() * w.float()).to(torch.bfloat16)


@pytest.mark.parametrize("M,K,N", [(1, 4096, 6144), (5, 1024, 2048), (16, 4096, 4096), (17, 2048, 3072),
                                   (64, 4096, 6144), (64, 4096, 28672), (200, 1152, 1024), (20, 16512, 512)])
def test_rms_norm_linear_matches_the_two_calls(M, K, N):
    x, w, s = make_inputs(M, K, N, seed=M + K)
    g = (torch.rand(K, generator=torch.Generator().manual_seed(K)) * 2).to(torch.bfloat16)
    xd, wd, gd, sd = x.cuda(), ops.pack_weight(w.cuda()), g.cuda(), s.cuda()
    fused = ops.rms_norm_proj(xd, gd, EPS, wd, sd, N, K)
    two = ops.int8_linear_packed(ops.rms_norm(xd, gd, EPS), wd, sd, N, K)
    torch.cuda.synchronize()
    assert torch.equal(fused, two), f"M={M} K={K} N={N}: fused != rms_norm then projection"
    rows = list(range(0, M, max(1, M // 8)))
    xn = _norm_ref(x, g)
    check_parity(fused[rows], oracle_rows(xn.float(), w, s, rows), f"rms_norm_proj M={M} K={K} N={N}")
    assert ops.device_status() == _lib.LSE_OK


@pytest.mark.parametrize("M", [3, 16, 40, 64])
def test_rms_norm_gate_up_silu_matches_the_two_calls(M):
    K, I = 2048, 2560
    x, w, s = make_inputs(M, K, 2 * I, seed=7 * M)
    g = (torch.rand(K, generator=torch.Generator().manual_seed(M)) + 0.5).to(torch.bfloat16)
    order = ops.interleave_gate_up_rows(I).cuda()
    wd = ops.pack_weight(w.cuda()[order])
    sd = s.cuda()[order]
    xd, gd = x.cuda(), g.cuda()
    fused = ops.rms_norm_proj(xd, gd, EPS, wd, sd, I, K, silu=True)
    two = ops.int8_gate_up_silu_packed(ops.rms_norm(xd, gd, EPS), wd, sd, I, K)
    torch.cuda.synchronize()
    assert torch.equal(fused, two), f"M={M}: fused gate_up + SiLU != rms_norm then gate_up + SiLU"
    xn = _norm_ref(x, g)
    acc = oracle_rows(xn.float(), w, s, list(range(M)))
    ref = acc[:, :I] / (1.0 + np.exp(-acc[:, :I])) * acc[:, I:]
    check_parity(fused, ref, f"rms_norm_proj silu M={M}")


def test_rms_norm_proj_refusals():
    K, N = 256, 256
    wp = ops.pack_weight(torch.zeros(N, K, dtype=torch.int8, device="cuda"))
    s = torch.ones(N, device="cuda")
    g = torch.ones(K, dtype=torch.bfloat16, device="cuda")
    x = torch.zeros(4, K, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError, match="bf16"):
        ops.rms_norm_proj(x.half(), g, EPS, wp, s, N, K)
    with pytest.raises(ValueError, match="norm_weight"):
        ops.rms_norm_proj(x, g[:128], EPS, wp, s, N, K)
    lib = _lib.load()
    y = torch.empty(4, N, dtype=torch.bfloat16, device="cuda")
    ws = torch.empty(int(lib.lse_int8_rms_norm_proj_workspace(4, K)), dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    # workspace too small, negative eps, I not a multiple of 8: refused before any launch
    assert lib.lse_int8_rms_norm_linear_packed(x.data_ptr(), 4, K, K, g.data_ptr(), EPS, wp.data_ptr(), s.data_ptr(),
                                               N, y.data_ptr(), N, ws.data_ptr(), 16, stream) == _lib.LSE_ERR_WORKSPACE
    assert lib.lse_int8_rms_norm_linear_packed(x.data_ptr(), 4, K, K, g.data_ptr(), -1.0, wp.data_ptr(), s.data_ptr(),
                                               N, y.data_ptr(), N, ws.data_ptr(), ws.numel(),
                                               stream) == _lib.LSE_ERR_INVALID_ARG
    assert lib.lse_int8_rms_norm_gate_up_silu_packed(x.data_ptr(), 4, K, K, g.data_ptr(), EPS, wp.data_ptr(),
                                                     s.data_ptr(), 124, y.data_ptr(), N, ws.data_ptr(), ws.numel(),
                                                     stream) == _lib.LSE_ERR_UNSUPPORTED
