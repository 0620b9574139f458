"""The torch.library operators `lse::int8_linear` and `lse::gate_up_silu` (liblse_torch.so, C++
over the C ABI) in bf16 and fp16, against the fp64 oracle on the same inputs: every kernel the
automatic choice reaches (decode kernel up to 16 tokens and, for weights of at most 32 MiB,
up to 32; tensor-core kernel above, both tile and schedule families), the fused residual add, the fused gate/up + SiLU, the int8 modules
dispatching to them natively in fp16, and the host-side refusals before any launch.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from llm_serving_engine_b200 import ops
from llm_serving_engine_b200.inputs import make_inputs
from llm_serving_engine_b200.int8_linear import Int8Linear, Int8LlamaMLP
from tests.gpu_helpers import check_parity, oracle_rows

pytestmark = pytest.mark.gpu

DTYPES = [torch.bfloat16, torch.float16]


def _case(M, K, N, dtype, seed):
    x, w, s = make_inputs(M, K, N, seed=seed)
    x = x.to(dtype)  # the oracle reads the same (rounded) values
    dev = torch.device("cuda")
    return x, w, s, x.to(dev), ops.pack_weight(w.to(dev)), s.to(dev)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("M", [1, 5, 16, 17, 32, 64, 300])
def test_int8_linear_op(M, dtype):
    K, N = 2048, 3072
    x, w, s, xd, wp, sd = _case(M, K, N, dtype, seed=M)
    lse = ops.torch_ops()
    y = lse.int8_linear(xd, wp, sd, N, K)
    assert y.dtype == dtype and y.shape == (M, N)
    check_parity(y, oracle_rows(x.float(), w, s, list(range(M))), f"lse::int8_linear {dtype} M={M}")
    # the same through the ctypes path
    y2 = ops.int8_linear_packed(xd, wp, sd, N, K)
    assert torch.equal(y, y2)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("M", [3, 40, 257])
def test_int8_linear_op_residual_and_leading_dims(M, dtype):
    K, N = 1024, 2048
    x, w, s, xd, wp, sd = _case(M, K, N, dtype, seed=100 + M)
    r = (torch.randn(M, N, generator=torch.Generator().manual_seed(M)) * 4).to(dtype)
    lse = ops.torch_ops()
    y = lse.int8_linear(xd.view(1, M, K), wp, sd, N, K, r.cuda().view(1, M, N))
    assert y.shape == (1, M, N) and y.dtype == dtype
    ref = oracle_rows(x.float(), w, s, list(range(M))) + r.double().numpy()
    check_parity(y[0], ref, f"lse::int8_linear residual {dtype} M={M}")


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("M", [4, 16, 64, 200])
def test_gate_up_silu_op(M, dtype):
    K, I = 1024, 1536
    x, w, s, xd, _, sd = _case(M, K, 2 * I, dtype, seed=7 + M)
    order = ops.interleave_gate_up_rows(I).cuda()
    wp = ops.pack_weight(w.cuda()[order])
    h = ops.torch_ops().gate_up_silu(xd, wp, sd[order], I, K)
    assert h.dtype == dtype and h.shape == (M, I)
    acc = oracle_rows(x.float(), w, s, list(range(M)))
    ref = acc[:, :I] / (1.0 + np.exp(-acc[:, :I])) * acc[:, I:]
    check_parity(h, ref, f"lse::gate_up_silu {dtype} M={M}")


def test_modules_run_fp16_natively():
    torch.manual_seed(0)
    lin = torch.nn.Linear(512, 768, bias=False).cuda().half()
    q = Int8Linear.from_linear(lin)
    x = torch.randn(3, 7, 512, device="cuda", dtype=torch.float16)
    y = q(x)
    assert y.dtype == torch.float16 and y.shape == (3, 7, 768)
    ref = x.float() @ q.dequantized(torch.float32).T
    assert ((y.float() - ref).abs().max() / ref.abs().max()).item() < 1e-2

    class _MLP(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.gate_proj = torch.nn.Linear(512, 1024, bias=False)
            self.up_proj = torch.nn.Linear(512, 1024, bias=False)
            self.down_proj = torch.nn.Linear(1024, 512, bias=False)

    mlp = Int8LlamaMLP.from_mlp(_MLP().cuda().half())
    out = mlp(x)
    assert out.dtype == torch.float16
    g = x.float() @ mlp.gate_weight().T
    u = x.float() @ mlp.up_weight().T
    ref = (torch.nn.functional.silu(g) * u) @ mlp.down_proj.dequantized(torch.float32).T
    assert ((out.float() - ref).abs().max() / ref.abs().max()).item() < 2e-2


def test_host_checks_refuse_before_launch():
    lse = ops.torch_ops()
    K, N = 256, 256
    wp = ops.pack_weight(torch.zeros(N, K, dtype=torch.int8, device="cuda"))
    s = torch.ones(N, device="cuda")
    with pytest.raises(RuntimeError, match="bfloat16 or float16"):
        lse.int8_linear(torch.zeros(2, K, device="cuda"), wp, s, N, K)
    with pytest.raises(RuntimeError, match="last dim"):
        lse.int8_linear(torch.zeros(2, K + 16, device="cuda", dtype=torch.bfloat16), wp, s, N, K)
    with pytest.raises(RuntimeError, match="packed int8 buffer"):
        lse.int8_linear(torch.zeros(2, K, device="cuda", dtype=torch.bfloat16), wp[:-16], s, N, K)
    with pytest.raises(RuntimeError, match="multiple of 8"):
        lse.gate_up_silu(torch.zeros(2, K, device="cuda", dtype=torch.bfloat16), wp, s[:248], 124, K)
