"""The reference engine's CPU path for a projection, restated for timing.

The reference runs every projection as a CPU `torch.nn.Linear` on its `_forward_hf` path
(`src/llm_serving_engine/model/model_runner.py:185-200`; linears reached at `:322-324`,
`:369`, `:223`).  It has no int8 variant (`model_runner.py:45-46` raises), so the closest
thing a user of the reference runs for an int8-quantized checkpoint is that `nn.Linear` on the
dequantized weight `W = q * s[:, None]`, dequantized once at load: `F.linear(x, W)` in the
model dtype.  The reference's CPU tests load float32 (`tests/factories.py:50-53` loads
`dtype="float32"`), so float32 is the default here.

Used only by bench.py's CPU baseline / reference arm and by tests: test infrastructure, not
the shipped path.
"""

from __future__ import annotations

import os
import platform

import torch
import torch.nn.functional as F


class ReferenceCpuLinear:
    """`nn.Linear(K, N, bias=False)` holding the dequantized int8 weight, on the CPU."""

    def __init__(self, q: torch.Tensor, s: torch.Tensor, dtype: torch.dtype = torch.float32):
        self.dtype = dtype
        self.weight = (q.float() * s.float()[:, None]).to(dtype).contiguous()

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        return F.linear(x.to(self.dtype), self.weight)


def host_threads() -> int:
    """Use every host core, as the reference's torch CPU path does by default."""
    n = os.cpu_count() or 1
    torch.set_num_threads(n)
    return torch.get_num_threads()


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return platform.processor() or "unknown"
