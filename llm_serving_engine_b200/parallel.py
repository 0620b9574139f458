"""Splits of the int8 linear over the ranks of a process group.

`y[:, n]` depends only on `W[n, :]`, `s[n]` and all of `x`, so a projection shards by output
rows with no reduction across ranks: rank r of g holds rows [r*N/g, (r+1)*N/g) of the int8
weight and their scales, `x` is replicated (every rank already holds its own copy of the
activation), and the only collective is an all-gather of the output shards, issued only where
the consumer needs the full output.  On B200 the collectives are NCCL over NVLink 5; the
shards' shapes keep each rank's kernel on the same configuration as a single-GPU call of N/g
rows.

* `ColumnParallelInt8Linear`: one projection split by output rows, shard-local kernel, and
  optionally the all-gather: `gather_output="shard_major"` returns the gathered shards as
  `[g, ..., N/g]` exactly as the collective leaves them (no copy); `True` reorders them into
  `[..., N]` (one more pass over the output).
* `RowParallelInt8Linear`: one projection split by input columns (K): rank r holds
  `W[:, K-block r]` and reads its block of x; the partial outputs (each with the full s[n])
  are summed by one all-reduce.
* `TensorParallelInt8MLP`: `down(silu(gate(x)) * up(x))` with gate_up split by output rows and
  down by input columns over the same intermediate blocks, so SiLU * mul stays local, the
  intermediate is never gathered, and the block's only collective is the all-reduce of its
  [..., H] output.  With the default (GPU) local linear and SiLU, the rank's gate and up rows
  are stored interleaved in 8-row blocks and gate_up + SiLU * mul is one fused launch;
  otherwise the rank's gate block precedes its up block and SiLU * mul runs after it.

The per-rank compute is `local_factory(q_rows, s_rows)`: by default an `Int8Linear` on this
rank's GPU (the sm_100a kernels; there is no CPU path).  Tests substitute a factory to run
the sharding and collective logic on CPU ranks.
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

__all__ = ["ColumnParallelInt8Linear", "RowParallelInt8Linear", "TensorParallelInt8MLP", "PeerWatch", "PeerLeft",
           "shard_rows",
           "interleaved_rows", "fused_rows", "gather_columns", "all_reduce_sum"]


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


def gather_columns(y: torch.Tensor, group=None, layout: str = "row_major") -> torch.Tensor:
    """All-gather the ranks' column shards `y [..., n]` (rank order).  layout "shard_major":
    `[world, ..., n]`, the collective's own output, no copy; "row_major": `[..., world * n]`,
    the shards reordered into full rows (a copy of the output, except when the leading dims
    hold one row)."""
    world, _ = _world(group)
    if layout not in ("row_major", "shard_major"):
        raise ValueError(f"gather_columns: layout must be 'row_major' or 'shard_major', got {layout!r}")
    lead, n = y.shape[:-1], y.shape[-1]
    if world == 1:
        return y.unsqueeze(0) if layout == "shard_major" else y
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
    if layout == "shard_major":
        return parts.view(world, *lead, n)
    return parts.permute(1, 0, 2).reshape(*lead, world * n)


def all_reduce_sum(y: torch.Tensor, group=None) -> torch.Tensor:
    """Sum `y` over the ranks of `group`, in place (NCCL on GPUs: on NVSwitch systems it may
    reduce inside the switch)."""
    world, _ = _world(group)
    if world > 1:
        dist.all_reduce(y, op=dist.ReduceOp.SUM, group=group)
    return y


class PeerLeft(RuntimeError):
    """A peer rank left (or stopped checking in) between steps."""

    def __init__(self, rank: int, why: str):
        super().__init__(f"rank {rank} {why}")
        self.rank = rank


class PeerWatch:
    """Failure detection on the host, between steps: before launching a step's collectives a
    rank checks in under the step number in the process group's key-value store and waits,
    bounded, until every peer has checked in.  A rank that stops says so (`leave`) before it
    goes.  A departed peer, or one that does not check in within `timeout_s`, raises `PeerLeft`
    on every other rank before any of its collectives is launched, so no GPU waits on a
    collective that cannot complete."""

    def __init__(self, store, rank: int, world: int, timeout_s: float = 5.0, prefix: str = "lse"):
        self.store, self.rank, self.world = store, rank, world
        self.timeout_s, self.prefix = timeout_s, prefix

    @classmethod
    def for_default_group(cls, timeout_s: float = 5.0) -> "PeerWatch":
        from torch.distributed import distributed_c10d as c10d

        return cls(c10d._get_default_store(), dist.get_rank(), dist.get_world_size(), timeout_s)

    def step(self, n: int) -> None:
        import time

        self.store.set(f"{self.prefix}/alive/{n}/{self.rank}", "1")
        deadline = time.monotonic() + self.timeout_s
        for r in range(self.world):
            if r == self.rank:
                continue
            while True:
                if self.store.check([f"{self.prefix}/left/{r}"]):
                    raise PeerLeft(r, f"left before step {n}")
                if self.store.check([f"{self.prefix}/alive/{n}/{r}"]):
                    break
                if time.monotonic() > deadline:
                    raise PeerLeft(r, f"did not check in for step {n} within {self.timeout_s} s")
                time.sleep(0.005)

    def leave(self) -> None:
        self.store.set(f"{self.prefix}/left/{self.rank}", "1")


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
        if not self.gather_output:
            return y
        return gather_columns(y, self.group, "shard_major" if self.gather_output == "shard_major" else "row_major")

    def extra_repr(self) -> str:
        world, rank = _world(self.group)
        return (f"in_features={self.in_features}, out_features={self.out_features}, rank {rank} of {world}, "
                f"gather_output={self.gather_output}")


class RowParallelInt8Linear(nn.Module):
    """The int8 linear with its input columns (K) split over the ranks of `group`: rank r holds
    `W[:, K-block r]` with the full scales and takes x's block r; the partial outputs are summed
    across the ranks (one all-reduce), or left to the caller with `reduce_output=False`."""

    def __init__(self, local: LocalLinear, in_features: int, out_features: int, group=None,
                 reduce_output: bool = True):
        super().__init__()
        self.local = local
        self.in_features = in_features  # full K across the group
        self.out_features = out_features
        self.group = group
        self.reduce_output = reduce_output

    @classmethod
    def from_quantized(cls, q: torch.Tensor, s: torch.Tensor, group=None, reduce_output: bool = True,
                       local_factory: LocalFactory = _default_local) -> "RowParallelInt8Linear":
        """Shard the full int8 weight `q [N, K]` (identical on every rank) by columns: keep this
        rank's contiguous K block and every scale."""
        world, rank = _world(group)
        N, K = q.shape
        cols = shard_rows(K, world, rank).to(q.device)
        local = local_factory(q.index_select(1, cols).contiguous(), s.contiguous())
        return cls(local, K, N, group, reduce_output)

    def forward(self, x_block: torch.Tensor) -> torch.Tensor:
        y = self.local(x_block)
        return all_reduce_sum(y, self.group) if self.reduce_output else y

    def extra_repr(self) -> str:
        world, rank = _world(self.group)
        return (f"in_features={self.in_features}, out_features={self.out_features}, rank {rank} of {world}, "
                f"reduce_output={self.reduce_output}")


class TensorParallelInt8MLP(nn.Module):
    """`down(act(gate(x)) * up(x))` with gate_up split by output rows and down by input
    columns over the same intermediate blocks: one all-reduce of the output, nothing gathered."""

    def __init__(self, gate_up: ColumnParallelInt8Linear, down: RowParallelInt8Linear, intermediate: int,
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
        down = RowParallelInt8Linear.from_quantized(q_down, s_down, group, local_factory=local_factory)
        return cls(gate_up, down, intermediate, group, act, fused=fused)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        world, _ = _world(self.group)
        i_local = self.intermediate_size // world
        if self.fused:
            lin = self.gate_up.local
            h_local = ops.torch_ops().gate_up_silu(x, lin.weight_packed, lin.scale, i_local, lin.in_features)
        else:
            gu = self.gate_up(x)  # [..., 2 * I / world]: this rank's gate block, then its up block
            gate, up = gu.split(i_local, dim=-1)
            h_local = self.act(gate) * up
        return self.down_proj(h_local)  # this rank's intermediate block -> partial sums -> all-reduce
