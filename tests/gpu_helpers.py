"""Shared helpers for the GPU tests: drive the C ABI directly (ctypes) on torch-allocated
device buffers and compare with the CPU oracle."""

from __future__ import annotations

import numpy as np
import torch

from llm_serving_engine_b200 import _lib
from oracle.ref_linear import parity_errors, ref_int8_linear


class Workspace:
    """Scratch for the C ABI's linear calls, grown to each call's need, plus a guard band after
    the needed bytes to catch overruns.  The library requires nothing of its contents; the
    buffer is filled with garbage (0xA5) so that a call relying on zeroed memory would fail."""

    GUARD = 4096

    def __init__(self, device="cuda"):
        self.device = device
        self.nbytes = 0
        self.buf = torch.full((self.GUARD,), 0xA5, dtype=torch.uint8, device=device)

    def ensure(self, M: int, K: int, N: int) -> "Workspace":
        need = int(_lib.load().lse_int8_linear_workspace(M, K, N))
        if need > self.nbytes:
            self.nbytes = need
            self.buf = torch.full((need + self.GUARD,), 0xA5, dtype=torch.uint8, device=self.device)
        return self

    @property
    def ptr(self) -> int:
        return self.buf.data_ptr()

    def counters_clear(self) -> bool:
        """Every stream-K counter a call used is back at zero (the last arriver re-arms it);
        counters no call used still hold the fill pattern."""
        head = self.buf[:_lib.WS_COUNTER_BYTES]
        return bool(((head == 0) | (head == 0xA5)).all().item())

    def guard_intact(self) -> bool:
        return bool((self.buf[self.nbytes:] == 0xA5).all().item())


def abi_linear(x: torch.Tensor, w: torch.Tensor, s: torch.Tensor, ws: Workspace, algo: int = 0,
               ldx: int | None = None, y: torch.Tensor | None = None, ldy: int | None = None) -> torch.Tensor:
    """Call lse_int8_linear_ex through ctypes. x: bf16 [M, >=K] (row stride ldx)."""
    lib = _lib.load()
    M = x.shape[0]
    N, K = w.shape
    ldx = x.stride(0) if ldx is None else ldx
    ws.ensure(M, K, N)
    if y is None:
        y = torch.empty((M, N), dtype=torch.bfloat16, device=x.device)
    ldy = y.stride(0) if ldy is None else ldy
    rc = lib.lse_int8_linear_ex(x.data_ptr(), M, K, ldx, w.data_ptr(), s.data_ptr(), N, y.data_ptr(), ldy,
                                ws.ptr, ws.nbytes, algo, torch.cuda.current_stream().cuda_stream)
    _lib.check(rc, "lse_int8_linear_ex")
    return y


def oracle_rows(x_cpu: torch.Tensor, w_cpu: torch.Tensor, s_cpu: torch.Tensor, rows, chunk: int = 4096) -> np.ndarray:
    """The fp64 oracle on the listed rows of x; the weight is widened `chunk` output rows at a
    time, so a 70B-sized matrix never exists in float64 at once."""
    xr = x_cpu[rows].float().numpy()
    w, s = w_cpu.numpy(), s_cpu.numpy()
    N = w.shape[0]
    if N <= chunk:
        return ref_int8_linear(xr, w, s)
    return np.concatenate([ref_int8_linear(xr, w[i:i + chunk], s[i:i + chunk]) for i in range(0, N, chunk)], axis=-1)


def check_parity(y_gpu: torch.Tensor, ref: np.ndarray, what: str = "") -> float:
    y = y_gpu.float().cpu().numpy()
    nw, ok, ratio = parity_errors(y, ref)
    assert np.all(np.isfinite(y)), f"{what}: non-finite output"
    assert nw <= 1e-2, f"{what}: normwise error {nw:.3e} > 1e-2"
    assert ok, f"{what}: elementwise criterion violated (worst ratio {ratio:.3f})"
    return nw
