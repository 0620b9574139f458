"""The splits over NCCL ranks on real GPUs (one process per GPU, 2 GPUs).

Each rank runs the sm_100a kernel on its row block and the shards are all-gathered over
NVLink (row-major, and shard-major as the collective leaves them); the result is compared
with the unsplit single-GPU projection (same kernel family, different shape, so within the
parity tolerance rather than bit for bit) and with the oracle.  The tensor-parallel MLP
(gate_up split by rows, down by input columns, one all-reduce) is compared with the unsplit
MLP arithmetic on one GPU.  Skipped when fewer than two GPUs are visible (a one-GPU run of
the suite).
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
import torch.nn.functional as F

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]

WORLD = 2


def _free_port() -> int:
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


def _case(rank: int, world: int) -> None:
    from llm_serving_engine_b200 import ops
    from llm_serving_engine_b200.inputs import make_inputs
    from llm_serving_engine_b200.int8_linear import Int8Linear
    from llm_serving_engine_b200.parallel import ColumnParallelInt8Linear, TensorParallelInt8MLP
    from oracle.ref_linear import parity_errors, ref_int8_linear

    dev = torch.device("cuda", rank)
    # projections: decode (skinny kernel) and prefill-sized (tensor-core kernel) token counts
    for M, K, N in [(4, 4096, 8192), (64, 4096, 4096), (300, 2048, 2048)]:
        x, w, s = make_inputs(M, K, N, seed=M + N)
        xd = x.to(dev)
        mod = ColumnParallelInt8Linear.from_quantized(w.to(dev), s.to(dev))
        y = mod(xd)
        torch.cuda.synchronize(dev)
        rows = np.array([0, M // 2, M - 1])
        ref = ref_int8_linear(x[rows].float().numpy(), w.numpy(), s.numpy())
        nw, ok, _ = parity_errors(y[torch.as_tensor(rows, device=dev)].float().cpu().numpy(), ref)
        assert nw <= 1e-2 and ok, (M, K, N, nw)
        single = Int8Linear.from_quantized(w.to(dev), s.to(dev))(xd)
        nw2, ok2, _ = parity_errors(y.float().cpu().numpy(), single.float().cpu().numpy().astype(np.float64))
        assert nw2 <= 1e-2 and ok2, (M, K, N, nw2)
        sm = ColumnParallelInt8Linear.from_quantized(w.to(dev), s.to(dev), gather_output="shard_major")(xd)
        assert sm.shape == (world, M, N // world)
        assert torch.equal(sm.permute(1, 0, 2).reshape(M, N), y)
    # tensor-parallel MLP vs the unsplit MLP arithmetic on one GPU
    H, I, M = 1024, 4096, 8
    g = torch.Generator().manual_seed(9)
    wg, wu, wdn = (torch.randn(*shape, generator=g) * 0.02 for shape in [(I, H), (I, H), (H, I)])
    qs = [ops.quantize_per_channel(t.to(dev)) for t in (wg, wu, wdn)]
    x = torch.randn(M, H, generator=g).to(torch.bfloat16).to(dev)
    mlp = TensorParallelInt8MLP.from_quantized(qs[0][0], qs[0][1], qs[1][0], qs[1][1], qs[2][0], qs[2][1])
    y = mlp(x)
    gu = Int8Linear.from_quantized(torch.cat([qs[0][0], qs[1][0]]), torch.cat([qs[0][1], qs[1][1]]))(x)
    ref = Int8Linear.from_quantized(*qs[2])(F.silu(gu[:, :I]) * gu[:, I:])
    # normwise only: each rank runs gate_up + SiLU * mul fused (fp32 intermediate, one bf16
    # rounding), the unsplit reference rounds gate, up and SiLU to bf16 separately
    nw, _, _ = parity_errors(y.float().cpu().numpy(), ref.float().cpu().numpy().astype(np.float64))
    assert mlp.fused and nw <= 1e-2, nw
    assert ops.device_status(dev) == 0


def _worker(rank: int, world: int, port: int) -> None:
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            device_id=torch.device("cuda", rank))
    try:
        _case(rank, world)
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_column_split_over_nccl_matches_single_gpu():
    if torch.cuda.device_count() < WORLD:
        pytest.skip(f"needs {WORLD} GPUs")
    mp.spawn(_worker, args=(WORLD, _free_port()), nprocs=WORLD, join=True)


def _leaving_worker(rank: int, world: int, port: int, out) -> None:
    """Step 0 over NCCL with every rank; then the last rank leaves with no collective in
    flight, and the others learn it on the host (PeerWatch) before launching step 1's."""
    import datetime
    import time

    from llm_serving_engine_b200.inputs import make_inputs
    from llm_serving_engine_b200.parallel import ColumnParallelInt8Linear, PeerLeft, PeerWatch

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            device_id=dev, timeout=datetime.timedelta(seconds=20))
    try:
        x, w, s = make_inputs(8, 1024, 2048, seed=3)
        mod = ColumnParallelInt8Linear.from_quantized(w.to(dev), s.to(dev))
        watch = PeerWatch.for_default_group(timeout_s=5.0)
        watch.step(0)
        y = mod(x.to(dev))
        torch.cuda.synchronize(dev)  # step 0's gather is complete on this rank
        if rank == world - 1:
            watch.leave()
            out.put((rank, "left"))
            return
        t0 = time.time()
        try:
            watch.step(1)
            mod(x.to(dev))
            out.put((rank, "completed"))
        except PeerLeft as e:
            out.put((rank, f"PeerLeft {e.rank} after {time.time() - t0:.2f} s, step 0 {tuple(y.shape)}"))
    finally:
        dist.destroy_process_group()


def test_rank_leaving_between_steps_is_reported_before_the_next_collective():
    """The NCCL form of the host-side failure test: no GPU waits on a collective that cannot
    complete, because the surviving rank raises PeerLeft from the store check before launching
    it (NVLS off, plain NCCL)."""
    if torch.cuda.device_count() < WORLD:
        pytest.skip(f"needs {WORLD} GPUs")
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_leaving_worker, args=(r, WORLD, port, out)) for r in range(WORLD)]
    for p in procs:
        p.start()
    results = dict(out.get(timeout=180) for _ in range(WORLD))
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
            pytest.fail("a rank hung")
    assert results[WORLD - 1] == "left"
    assert results[0].startswith(f"PeerLeft {WORLD - 1} after"), results
