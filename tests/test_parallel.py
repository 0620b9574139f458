"""Splits over ranks (llm_serving_engine_b200.parallel) on CPU gloo ranks.

The per-rank kernel is replaced by the oracle (a `local_factory` returning bf16-rounded fp64
results), so these tests check what the splits themselves must get right - which rows and
columns each rank holds, the gate/up interleave, the all-gather and its column order (row-major
and shard-major), the all-reduce of the K split, leading dimensions - at world sizes 2 and 4:
the output-row split bit for bit against the unsplit computation; the K split (partials
rounded to bf16 and summed) within the parity tolerance of the fp64 computation, identical on
every rank.  The GPU run of the same modules over NCCL is tests/test_gpu_multi.py.
"""

from __future__ import annotations

import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
import torch.nn.functional as F

from llm_serving_engine_b200.parallel import (ColumnParallelInt8Linear, RowParallelInt8Linear,
                                              TensorParallelInt8MLP, fused_rows, gather_columns, interleaved_rows,
                                              shard_rows)
from oracle.ref_linear import ref_int8_linear, ref_quantize


def oracle_local(q: torch.Tensor, s: torch.Tensor):
    qn, sn = q.numpy(), s.numpy()

    def run(x: torch.Tensor) -> torch.Tensor:
        y = ref_int8_linear(x.reshape(-1, x.shape[-1]).float().numpy(), qn, sn)
        return torch.from_numpy(y).to(torch.bfloat16).reshape(*x.shape[:-1], qn.shape[0])

    return run


def _weights(seed: int, N: int, K: int):
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(N, K, generator=g) * torch.rand(N, 1, generator=g)
    q, s = ref_quantize(w.numpy())
    return torch.from_numpy(q), torch.from_numpy(s)


def _x(seed: int, *shape):
    return torch.randn(*shape, generator=torch.Generator().manual_seed(seed)).to(torch.bfloat16)


def _column_case(rank: int, world: int) -> None:
    M, K, N = 5, 64, 48
    q, s = _weights(1, N, K)
    x = _x(2, M, K)
    full = oracle_local(q, s)(x)
    mod = ColumnParallelInt8Linear.from_quantized(q, s, local_factory=oracle_local)
    y = mod(x)
    assert y.shape == (M, N) and torch.equal(y, full)
    # without the gather each rank keeps its own contiguous block
    part = ColumnParallelInt8Linear.from_quantized(q, s, gather_output=False, local_factory=oracle_local)(x)
    n = N // world
    assert torch.equal(part, full[:, rank * n:(rank + 1) * n])
    # any leading shape
    x3 = _x(3, 2, 3, K)
    assert torch.equal(mod(x3), oracle_local(q, s)(x3))
    # shard-major: the collective's [world, ..., n] as it is
    sm = ColumnParallelInt8Linear.from_quantized(q, s, gather_output="shard_major", local_factory=oracle_local)(x3)
    full3 = oracle_local(q, s)(x3)
    assert sm.shape == (world, 2, 3, n)
    for r in range(world):
        assert torch.equal(sm[r], full3[..., r * n:(r + 1) * n])


def _rel_err(y: torch.Tensor, ref: np.ndarray) -> float:
    return float(np.abs(y.double().numpy() - ref).max() / np.abs(ref).max())


def _same_on_every_rank(y: torch.Tensor, world: int) -> None:
    ys = [torch.empty_like(y) for _ in range(world)]
    dist.all_gather(ys, y.contiguous())
    assert all(torch.equal(t, ys[0]) for t in ys)


def _row_case(rank: int, world: int) -> None:
    M, K, N = 4, 128, 40
    q, s = _weights(11, N, K)
    x = _x(12, 1, M, K)
    k = K // world
    mod = RowParallelInt8Linear.from_quantized(q, s, local_factory=oracle_local)
    y = mod(x[..., rank * k:(rank + 1) * k])
    assert y.shape == (1, M, N)
    ref = ref_int8_linear(x.reshape(M, K).float().numpy().astype(np.float64), q.numpy(), s.numpy())
    assert _rel_err(y.reshape(M, N), ref) <= 1e-2
    _same_on_every_rank(y, world)


def _mlp_case(rank: int, world: int) -> None:
    H, I, M = 32, 64, 3
    qg, sg = _weights(4, I, H)
    qu, su = _weights(5, I, H)
    qd, sd = _weights(6, H, I)
    x = _x(7, M, H)
    # the unsplit computation in fp64
    x64 = x.float().numpy().astype(np.float64)
    g = ref_int8_linear(x64, qg.numpy(), sg.numpy())
    u = ref_int8_linear(x64, qu.numpy(), su.numpy())
    ref = ref_int8_linear(g / (1.0 + np.exp(-g)) * u, qd.numpy(), sd.numpy())
    mlp = TensorParallelInt8MLP.from_quantized(qg, sg, qu, su, qd, sd, local_factory=oracle_local)
    assert not mlp.fused  # a substituted local linear keeps gate block | up block and SiLU * mul after it
    assert isinstance(mlp.down_proj, RowParallelInt8Linear)
    y = mlp(x)
    assert y.shape == (M, H)
    assert _rel_err(y, ref) <= 2e-2
    _same_on_every_rank(y, world)


def _gather_order_case(rank: int, world: int) -> None:
    y = torch.full((2, 3), float(rank), dtype=torch.bfloat16)
    out = gather_columns(y)
    expect = torch.cat([torch.full((2, 3), float(r), dtype=torch.bfloat16) for r in range(world)], dim=1)
    assert torch.equal(out, expect)


def _worker(rank: int, world: int, port: int, case) -> None:
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        case(rank, world)
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _free_port() -> int:
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


def _run(case, world: int) -> None:
    mp.spawn(_worker, args=(world, _free_port(), case), nprocs=world, join=True)


@pytest.mark.parametrize("world", [2, 4])
def test_column_split_matches_unsplit(world):
    _run(_column_case, world)


@pytest.mark.parametrize("world", [2, 4])
def test_tensor_parallel_mlp_matches_unsplit(world):
    _run(_mlp_case, world)


def test_gather_puts_rank_blocks_in_order():
    _run(_gather_order_case, 2)


@pytest.mark.parametrize("world", [2, 4])
def test_row_split_matches_unsplit(world):
    _run(_row_case, world)


def test_row_assignment():
    assert torch.equal(shard_rows(12, 3, 1), torch.arange(4, 8))
    assert torch.equal(interleaved_rows(8, 2, 1), torch.tensor([4, 5, 6, 7, 12, 13, 14, 15]))
    # every row exactly once across the ranks
    rows = torch.cat([interleaved_rows(8, 4, r) for r in range(4)])
    assert sorted(rows.tolist()) == list(range(16))
    with pytest.raises(ValueError):
        shard_rows(10, 4, 0)
    assert np.array_equal(np.concatenate([shard_rows(12, 4, r).numpy() for r in range(4)]), np.arange(12))


# ---- a rank that fails: the others end with an error, not a hang ----------------------
def _failing_rank_worker(rank: int, world: int, port: int, out) -> None:
    import datetime
    import time

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=3))
    try:
        q, s = _weights(1, 48, 64)
        mod = ColumnParallelInt8Linear.from_quantized(q, s, local_factory=oracle_local)
        if rank == world - 1:
            out.put((rank, "left before the collective"))
            return  # this rank fails between steps: it never joins the gather
        t0 = time.time()
        try:
            mod(_x(2, 5, 64))
            out.put((rank, "completed"))
        except Exception as e:  # noqa: BLE001 - any backend error is the expected outcome
            out.put((rank, f"error after {time.time() - t0:.1f} s: {type(e).__name__}"))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_rank_leaving_before_the_gather_errors_the_others(world):
    """Failure on the host, as on a GPU pool: one rank leaves between steps; the others' next
    collective ends with an error within the process group's short timeout instead of hanging."""
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_rank_worker, args=(r, world, port, out)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(out.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
            pytest.fail("a rank hung")
    assert results[world - 1] == "left before the collective"
    for r in range(world - 1):
        assert results[r].startswith("error after"), results


def test_fused_rows_interleave_the_rank_block_in_8_row_blocks():
    """Rank r's gate and up rows in the fused kernel's order: 8 gate rows, then the matching
    8 up rows; the same set of rows as the unfused order."""
    I, world = 32, 2
    for rank in range(world):
        f = fused_rows(I, world, rank)
        base = rank * I // world
        expect = [base + j for j in range(8)] + [I + base + j for j in range(8)] + \
                 [base + 8 + j for j in range(8)] + [I + base + 8 + j for j in range(8)]
        assert f.tolist() == expect
        assert sorted(f.tolist()) == sorted(interleaved_rows(I, world, rank).tolist())
    with pytest.raises(ValueError):
        fused_rows(24, 2, 0)  # 12 rows per rank


# ---- the same failure detected on the host before any collective (PeerWatch) -----------
def _watched_worker(rank: int, world: int, port: int, out) -> None:
    import datetime
    import time

    from llm_serving_engine_b200.parallel import PeerLeft, PeerWatch

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=30))
    try:
        q, s = _weights(1, 48, 64)
        mod = ColumnParallelInt8Linear.from_quantized(q, s, local_factory=oracle_local)
        watch = PeerWatch.for_default_group(timeout_s=5.0)
        watch.step(0)
        y = mod(_x(2, 5, 64))  # step 0: every rank present
        if rank == world - 1:
            watch.leave()
            out.put((rank, "left after step 0"))
            return
        t0 = time.time()
        try:
            watch.step(1)
            mod(_x(2, 5, 64))
            out.put((rank, "completed"))
        except PeerLeft as e:
            out.put((rank, f"PeerLeft {e.rank} after {time.time() - t0:.2f} s; step 0 shape {tuple(y.shape)}"))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_peer_watch_reports_a_departed_rank_before_the_collective(world):
    """The last rank leaves after a completed step; every other rank learns it from the store at
    its next check-in and raises PeerLeft at once, long before the process group's 30 s timeout,
    without launching the step's collective."""
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_watched_worker, args=(r, world, port, out)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(out.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
            pytest.fail("a rank hung")
    assert results[world - 1] == "left after step 0"
    for r in range(world - 1):
        assert results[r].startswith(f"PeerLeft {world - 1} after"), results
        assert float(results[r].split("after ")[1].split(" s")[0]) < 5.0
