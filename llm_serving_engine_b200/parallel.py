"""Output-column (N) split of the int8 linear over the ranks of a process group.

`y[:, n]` depends only on `W[n, :]`, `s[n]` and all of `x`, so the projections shard by
output rows with no reduction across ranks: rank r of g holds rows [r*N/g, (r+1)*N/g) of the
int8 weight and their scales, `x` is replicated (every rank already holds its own copy of
the activation), and the only collective is an all-gather of the output shards, issued
only where the consumer needs the full output (`gather_output`).  On B200 the gather is
NCCL over NVLink 5; the shards' shapes keep each rank's kernel on the same configuration as
a single-GPU call of N/g rows.

* `ColumnParallelInt8Linear`: one projection, shard-local kernel, optional all-gather.
* `TensorParallelInt8MLP`: `down(silu(gate(x)) * up(x))` with both projections N-split.
  Rank r holds the gate rows and the up rows of intermediate block r, so SiLU * mul stays
  local; the intermediate block is all-gathered once (down needs all of its K) and down's
  output block is gathered at the end.  With the default (GPU) local linear and SiLU, the
  rank's gate and up rows are stored interleaved in 8-row blocks and gate_up + SiLU * mul is
  one fused launch (`ops.int8_gate_up_silu_packed`); otherwise the rank's gate block
  precedes its up block and SiLU * mul runs after the projection.

The per-rank compute is `local_factory(q_rows, s_rows)`: by default an `Int8Linear` on this
rank's GPU (the sm_100a kernels; there is no CPU path).  Tests substitute a factory to run
the sharding and gather logic on CPU ranks.
"""

from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist
import torch.nn as nn
import torch.nn.functional as F

from . import ops
from .int8_linear import Int8Linear

LocalLinear = Callable[[torch.Tensor], torch.Tensor]
LocalFactory = Callable[[torch.Tensor, torch.Tensor], LocalLinear]

__all__ = ["ColumnParallelInt8Linear", "TensorParallelInt8MLP", "shard_rows", "interleaved_rows", "fused_rows",
           "gather_columns"]


def _default_local(q: torch.Tensor, s: torch.Tensor) -> LocalLinear:
    return Int8Linear.from_quantized(q, s)


def _world(group) -> tuple[int, int]:
    """(world size, rank) of `group`; a process without a process group is a world of one."""
    if not (dist.is_available() and dist.is_initialized()):
        return 1, 0
    return dist.get_world_size(group), dist.get_rank(group)


def shard_rows(N: int, world: int, rank: int) -> torch.Tensor:
    """Output rows of rank `rank`: the contiguous block [rank*N/world, (rank+1)*N/world)."""
    if N % world:
        raise ValueError(f"column split: N={N} is not a multiple of the {world} ranks")
    n = N // world
    return torch.arange(rank * n, (rank + 1) * n)


def interleaved_rows(intermediate: int, world: int, rank: int) -> torch.Tensor:
    """Rows of a fused [gate; up] weight (2 * intermediate rows) for rank `rank`: its gate
    block followed by the matching up block, so gate and up of the same intermediate
    columns land on the same rank."""
    blk = shard_rows(intermediate, world, rank)
    return torch.cat([blk, blk + intermediate])


def fused_rows(intermediate: int, world: int, rank: int) -> torch.Tensor:
    """The same rows as `interleaved_rows`, in the order the fused gate_up + SiLU * mul kernel
    reads: 8 gate rows of the rank's block, then the matching 8 up rows, and so on."""
    blk = shard_rows(intermediate, world, rank)
    if blk.numel() % 8:
        raise ValueError(f"fused gate/up rows: {blk.numel()} intermediate rows per rank is not a multiple of 8")
    b = blk.view(-1, 8)
    return torch.stack([b, b + intermediate], dim=1).reshape(-1)


def _is_silu(act) -> bool:
    # torch's SiLU, or transformers' SiLUActivation (ACT2FN["silu"])
    return act is F.silu or type(act).__name__ in ("SiLU", "SiLUActivation")


def gather_columns(y: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather the ranks' column shards `y [..., n]` into `[..., world * n]` (rank order)."""
    world, _ = _world(group)
    if world == 1:
        return y
    lead, n = y.shape[:-1], y.shape[-1]
    flat = y.reshape(-1, n).contiguous()
    rows = flat.shape[0]
    if dist.get_backend(group) == "nccl":
        out = torch.empty((world * rows, n), dtype=y.dtype, device=y.device)
        dist.all_gather_into_tensor(out, flat, group=group)
        parts = out.view(world, rows, n)
    else:
        chunks = [torch.empty_like(flat) for _ in range(world)]
        dist.all_gather(chunks, flat, group=group)
        parts = torch.stack(chunks)
    return parts.permute(1, 0, 2).reshape(*lead, world * n)


class ColumnParallelInt8Linear(nn.Module):
    """The int8 linear with its output rows split over the ranks of `group`."""

    def __init__(self, local: LocalLinear, in_features: int, out_features: int, group=None,
                 gather_output: bool = True):
        super().__init__()
        self.local = local
        self.in_features = in_features
        self.out_features = out_features  # full N across the group
        self.group = group
        self.gather_output = gather_output

    @classmethod
    def from_quantized(cls, q: torch.Tensor, s: torch.Tensor, group=None, gather_output: bool = True,
                       rows: torch.Tensor | None = None,
                       local_factory: LocalFactory = _default_local) -> "ColumnParallelInt8Linear":
        """Shard the full int8 weight `q [N, K]` and scales `s [N]` (identical on every rank):
        keep `rows` (default: this rank's contiguous block)."""
        world, rank = _world(group)
        N, K = q.shape
        if rows is None:
            rows = shard_rows(N, world, rank)
        rows = rows.to(q.device)
        local = local_factory(q.index_select(0, rows).contiguous(), s.index_select(0, rows).contiguous())
        return cls(local, K, N, group, gather_output)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        y = self.local(x)
        return gather_columns(y, self.group) if self.gather_output else y

    def extra_repr(self) -> str:
        world, rank = _world(self.group)
        return (f"in_features={self.in_features}, out_features={self.out_features}, rank {rank} of {world}, "
                f"gather_output={self.gather_output}")


class TensorParallelInt8MLP(nn.Module):
    """`down(act(gate(x)) * up(x))` with gate_up and down split over output rows."""

    def __init__(self, gate_up: ColumnParallelInt8Linear, down: ColumnParallelInt8Linear, intermediate: int,
                 group=None, act=F.silu, fused: bool = False):
        super().__init__()
        self.gate_up = gate_up
        self.down_proj = down
        self.intermediate_size = intermediate
        self.group = group
        self.act = act
        # fused: gate_up.local is an Int8Linear over `fused_rows` (8-row interleave)
        self.fused = fused

    @classmethod
    def from_quantized(cls, q_gate: torch.Tensor, s_gate: torch.Tensor, q_up: torch.Tensor, s_up: torch.Tensor,
                       q_down: torch.Tensor, s_down: torch.Tensor, group=None, act=F.silu,
                       local_factory: LocalFactory = _default_local) -> "TensorParallelInt8MLP":
        world, rank = _world(group)
        intermediate = q_gate.shape[0]
        if q_up.shape != q_gate.shape or q_down.shape[1] != intermediate:
            raise ValueError("TensorParallelInt8MLP: gate/up must be [I, H] and down [H, I]")
        q_gu = torch.cat([q_gate, q_up], dim=0)
        s_gu = torch.cat([s_gate, s_up], dim=0)
        if intermediate % world:
            raise ValueError(f"TensorParallelInt8MLP: intermediate size {intermediate} is not a multiple of {world}")
        fused = local_factory is _default_local and _is_silu(act) and (intermediate // world) % 8 == 0
        rows = fused_rows(intermediate, world, rank) if fused else interleaved_rows(intermediate, world, rank)
        gate_up = ColumnParallelInt8Linear.from_quantized(q_gu, s_gu, group, gather_output=False, rows=rows,
                                                          local_factory=local_factory)
        down = ColumnParallelInt8Linear.from_quantized(q_down, s_down, group, gather_output=True,
                                                       local_factory=local_factory)
        return cls(gate_up, down, intermediate, group, act, fused=fused)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        world, _ = _world(self.group)
        if self.fused:
            lin = self.gate_up.local
            h_local = ops.int8_gate_up_silu_packed(x.to(torch.bfloat16), lin.weight_packed, lin.scale,
                                                   self.intermediate_size // world, lin.in_features)
        else:
            gu = self.gate_up(x)  # [..., 2 * I / world]: this rank's gate block, then its up block
            gate, up = gu.split(self.intermediate_size // world, dim=-1)
            h_local = self.act(gate) * up
        h = gather_columns(h_local, self.group)  # [..., I]
        y = self.down_proj(h)
        return y.to(x.dtype) if self.fused and y.dtype != x.dtype else y
