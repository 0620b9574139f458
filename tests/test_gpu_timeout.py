"""The bounded waits of the tensor-core kernels give up, report, and leave the device usable.

A wait limit of one SM cycle (lse_set_wait_limit) makes every data wait of a tensor-core launch
that is not already satisfied at its first test give up: the CTA raises its abort flag, records
LSE_ERR_DEVICE_TIMEOUT, drains its own copies and MMAs under the default limit, frees its tensor
memory and returns.  Nothing faults, traps or hangs: the host reads the status, restores the
default limit, and the same call on the same stream is then correct (a CTA that left tensor
memory allocated would make that call's allocation wait forever, so its passing also shows the
memory was freed).  Every schedule of the kernel is covered: the thread-block-cluster split
(decode-sized M), data-parallel/stream-K tiles (prefill-sized M) and the fused gate/up + SiLU
epilogue.
"""

from __future__ import annotations

import pytest
import torch

from llm_serving_engine_b200 import _lib, ops
from llm_serving_engine_b200.inputs import make_inputs
from tests.gpu_helpers import check_parity, oracle_rows

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _restore_limit():
    yield
    ops.set_wait_limit(0)
    ops.device_status()


def _packed_case(M: int, K: int, N: int, seed: int):
    x, w, s = make_inputs(M, K, N, seed=seed)
    dev = torch.device("cuda")
    return x, w, s, x.to(dev), ops.pack_weight(w.to(dev)), s.to(dev)


@pytest.mark.parametrize("M,K,N", [(64, 4096, 6144), (512, 2048, 4096)])
def test_linear_timeout_reports_and_next_call_is_clean(M, K, N):
    x, w, s, xd, wp, sd = _packed_case(M, K, N, seed=40 + M)
    assert ops.device_status() == _lib.LSE_OK
    ops.set_wait_limit(1)
    ops.int8_linear_packed(xd, wp, sd, N, K, algo=ops.ALGO_TCGEN05)  # the launch itself succeeds
    assert ops.device_status() == _lib.LSE_ERR_DEVICE_TIMEOUT
    ops.set_wait_limit(0)
    assert ops.device_status() == _lib.LSE_OK  # cleared by the read above
    y = ops.int8_linear_packed(xd, wp, sd, N, K, algo=ops.ALGO_TCGEN05)
    assert ops.device_status() == _lib.LSE_OK
    rows = list(range(0, M, max(1, M // 16)))
    check_parity(y[rows], oracle_rows(x, w, s, rows), f"after timeout M={M}")


def test_gate_up_silu_timeout_reports_and_next_call_is_clean():
    M, K, I = 64, 2048, 2048
    x, w, s, xd, _, sd = _packed_case(M, K, 2 * I, seed=77)
    order = ops.interleave_gate_up_rows(I)
    wd = w.to("cuda")[order.to("cuda")]
    wp = ops.pack_weight(wd)
    so = sd[order.to("cuda")]
    ops.set_wait_limit(1)
    ops.int8_gate_up_silu_packed(xd, wp, so, I, K)
    assert ops.device_status() == _lib.LSE_ERR_DEVICE_TIMEOUT
    ops.set_wait_limit(0)
    h = ops.int8_gate_up_silu_packed(xd, wp, so, I, K)
    assert ops.device_status() == _lib.LSE_OK
    acc = xd.float() @ (w.to("cuda").float() * sd[:, None]).T
    ref = torch.nn.functional.silu(acc[:, :I]) * acc[:, I:]
    err = ((h.float() - ref).abs().max() / ref.abs().max()).item()
    assert err < 1e-2, f"fused gate/up after timeout: max error {err:.3e} of the largest output"
