#!/usr/bin/env python
"""Benchmark of the sm_100a int8 weight-only linear (one JSON line on rank 0).

Metric: int8 linear HBM GB/s (M<=64) & TFLOP/s (prefill) vs roofline;
decode tok/s.

Workload (`config.workload`): config 2, the decode sweep: M in {1, 4, 16, 64} x the four
Llama-3-8B projection shapes (K, N) = (4096, 6144) QKV, (4096, 4096) O, (4096, 28672)
gate_up, (14336, 4096) down.  One step = the int8 projections of one Llama-3-8B decode
iteration (32 layers x 4 projections, each layer with its own weights: 6.98 GB of int8, far
larger than L2) for each of the four M: 512 launches, captured once in a CUDA graph (the
reference engine replays decode iterations as CUDA graphs, decode_graph.py:87-140) and
replayed.  `value` = algorithmic bytes (N*K + 4N + 2MK + 2MN per launch) / device time.

Extra keys: `prefill` (config 3 sweep, TFLOP/s against the bf16 dense peak), `points`
(per-shape breakdown), `roofline` for the dominant kernel, `cpu_baseline` (the reference's
CPU path on the host cores), `e2e` (pinned host inputs copied in, graph replay, outputs
copied back, every step), `clocks` (nvidia-smi sampled during the timed region).

`--impl reference` times the reference's own CPU implementation of the path (the CPU
nn.Linear of `_forward_hf`, float32, on the dequantized weights; the reference has no int8
kernel) on a bounded sample of the same workload with all host threads.

Multi-GPU (`torchrun --nproc-per-node N bench.py --gpus N`): every rank holds its own
column stripe of an N-times-wider layer stack (the same per-rank shapes), no collective in
the data path; value = bytes all ranks processed / max over ranks of the device time
(weak scaling).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import torch
import torch.nn.functional as F

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

from llm_serving_engine_b200.inputs import (DECODE_M, LLAMA3_8B_SHAPES, LLAMA3_70B_SHAPES, PREFILL_M,  # noqa: E402
                                            linear_bytes, linear_flops)

METRIC = "int8 linear HBM GB/s (M<=64) & TFLOP/s (prefill) vs roofline; decode tok/s"
UNIT = "GB/s"
N_LAYERS = 32
SHAPE_ORDER = ("qkv", "o", "gate_up", "down")
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--layers", type=int, default=N_LAYERS)
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--no-70b", action="store_true", help="skip the Llama-3-70B column-split sweep (config 5)")
    ap.add_argument("--no-e2e-decode", action="store_true", help="skip the end-to-end model decode (config 4)")
    ap.add_argument("--no-engine-decode", action="store_true",
                    help="skip config 4 through the reference engine's ModelRunner (needs baseline/_ref)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=12.0, help="bounded CPU sample length")
    return ap.parse_args()


def peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "measured"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, 1400.0, "fallback"


def committed_traffic():
    """Per-launch DRAM bytes of the dominant kernel from the committed ncu summary."""
    path = os.path.join(REPO, "profiles", "traffic.json")
    try:
        with open(path) as f:
            return json.load(f)
    except (OSError, ValueError):
        return {}


# --------------------------------------------------------------------------------------
# clocks sampled during the timed region
class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.15)
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            time.sleep(0.1)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self):
        sms, maxes, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in getattr(self, "lines", []):
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sms.append(float(parts[1]))
                maxes.append(float(parts[2]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        if not sms:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sms), "sm_max_mhz": max(maxes), "reasons": sorted(reasons),
                "samples": len(sms)}


# --------------------------------------------------------------------------------------
def setup_dist(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def max_over_ranks(val: float, world: int) -> float:
    if world == 1:
        return val
    import torch.distributed as dist

    t = torch.tensor([val], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def make_weights(layers: int, device, seed: int, ops):
    """Per layer, per shape: int8 W uniform on [-127, 127] and fp32 s uniform [1e-4, 5e-4],
    drawn on the device from a seeded generator (7 GB would take minutes on the host), then
    repacked once into the tile-contiguous layout the module stores (Int8Linear)."""
    g = torch.Generator(device=device).manual_seed(seed)
    out = []
    for _ in range(layers):
        d = {}
        for name in SHAPE_ORDER:
            K, N = LLAMA3_8B_SHAPES[name]
            w = torch.randint(-127, 128, (N, K), generator=g, device=device, dtype=torch.int8)
            s = torch.empty(N, device=device).uniform_(1e-4, 5e-4, generator=g)
            d[name] = (ops.pack_weight(w), s)
            del w
        out.append(d)
    return out


def linear_call(ops, x, wp, s, y, name):
    K, N = LLAMA3_8B_SHAPES[name]
    ops.int8_linear_packed(x, wp, s, N, K, out=y)


def decode_step_fn(weights, xs, ys, ops):
    def step():
        for M in DECODE_M:
            for layer in weights:
                for name in SHAPE_ORDER:
                    wp, s = layer[name]
                    linear_call(ops, xs[(M, name)], wp, s, ys[(M, name)], name)
    return step


def capture(fn, warm_stream):
    warm_stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(warm_stream):
        fn()
    torch.cuda.current_stream().wait_stream(warm_stream)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=warm_stream):
        fn()
    torch.cuda.synchronize()
    return g


def time_graph(g, reps: int) -> float:
    """Average ms per replay, CUDA events on the replay stream, synchronized both sides."""
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        g.replay()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / reps


# --------------------------------------------------------------------------------------
TP_M = (1, 32, 256, 4096)


def tp70b_sweep(world: int, rank: int, dev, ops, warm):
    """Config 5: Llama-3-70B projection shapes with the output rows (N) split over the
    `world` ranks.  Per point (max over ranks): the rank's kernel time on its N/world rows
    (CUDA graph over rotated weight copies, so the weights come from HBM), the NCCL
    all-gather of the output shards into the shard-major [world, M, N/world] the collective
    produces (llm_serving_engine_b200.parallel.gather_columns, no reorder copy), and the end to
    end time of kernel + gather, each in a CUDA graph, CUDA events."""
    from llm_serving_engine_b200.parallel import gather_columns

    g = torch.Generator(device=dev).manual_seed(77 + rank)
    pts = []
    all_ok = True
    for name in SHAPE_ORDER:
        K, N = LLAMA3_70B_SHAPES[name]
        n = N // world
        copies = max(1, min(8, -(-3 * 126 * 2**20 // (n * K))))
        # the full weight, identical on every rank (common seed): copy 0 of the rotation is this
        # rank's row block of it, and the whole of it gives the single-GPU output the gathered
        # output is checked against; the other copies only rotate the weight reads past L2
        gf = torch.Generator(device=dev).manual_seed(1000 + K + N)
        w_full = torch.randint(-127, 128, (N, K), generator=gf, device=dev, dtype=torch.int8)
        s_full = torch.empty(N, device=dev).uniform_(1e-4, 5e-4, generator=gf)
        full_packed = ops.pack_weight(w_full)
        ws = [ops.pack_weight(w_full[rank * n:(rank + 1) * n])]
        del w_full
        for _ in range(copies - 1):
            w = torch.randint(-127, 128, (n, K), generator=g, device=dev, dtype=torch.int8)
            ws.append(ops.pack_weight(w))
            del w
        s = s_full[rank * n:(rank + 1) * n].contiguous()
        for M in TP_M:
            x = torch.randn(M, K, generator=gf, device=dev).to(torch.bfloat16)  # same x on every rank
            y = torch.empty(M, n, device=dev, dtype=torch.bfloat16)

            def one(x=x, y=y):
                for wp in ws:
                    ops.int8_linear_packed(x, wp, s, n, K, out=y)
            g1 = capture(one, warm)
            time_graph(g1, 2)
            t_k = time_graph(g1, 5) / copies
            del g1
            t_g = 0.0
            if world > 1:
                # the NCCL gather alone, and kernel + gather, each captured in a CUDA graph (as a
                # graphed decode step runs them); every rank captures the same sequence
                def gather10(y=y):
                    for _ in range(10):
                        gather_columns(y, layout="shard_major")
                g2 = capture(gather10, warm)
                time_graph(g2, 1)
                t_g = time_graph(g2, 3) / 10
                del g2

            def e2e10(x=x, y=y):
                for i in range(10):
                    ops.int8_linear_packed(x, ws[i % copies], s, n, K, out=y)
                    gather_columns(y, layout="shard_major")
            g3 = capture(e2e10, warm)
            time_graph(g3, 1)
            t_e = time_graph(g3, 3) / 10
            del g3
            # parity of the split: the gathered [M, N] output against one GPU's call on the whole
            # weight, on sampled rows, the same check on every rank (north_star tolerance)
            ops.int8_linear_packed(x, ws[0], s, n, K, out=y)
            full = gather_columns(y)
            rows = torch.unique(torch.tensor([0, M // 3, M // 2, M - 1], device=dev))
            ref = ops.int8_linear_packed(x[rows], full_packed, s_full, N, K).float()
            err = ((full[rows].float() - ref).abs().max() / ref.abs().max().clamp_min(1e-30)).item()
            ok = max_over_ranks(0.0 if err <= 1e-2 else 1.0, world) == 0.0
            all_ok = all_ok and ok
            t_k, t_g, t_e = (max_over_ranks(v, world) for v in (t_k, t_g, t_e))
            pts.append({"M": M, "shape": name, "K": K, "N": N, "rows_per_gpu": n,
                        "kernel_us": round(t_k * 1e3, 2), "gather_us": round(t_g * 1e3, 2),
                        "e2e_us": round(t_e * 1e3, 2),
                        "kernel_GBps_per_gpu": round(linear_bytes(M, K, n) / t_k / 1e6, 1),
                        "kernel_TFLOPs_per_gpu": round(linear_flops(M, K, n) / t_k / 1e9, 1),
                        "gather_bytes": M * N * 2 if world > 1 else 0,
                        "parity_vs_one_gpu": {"normwise": float(f"{max_over_ranks(err, world):.3e}"), "ok": ok}})
            del x, y, full, ref
        del ws, full_packed
        torch.cuda.empty_cache()
    if not all_ok:
        raise RuntimeError(f"config5 column split: gathered output differs from the one-GPU output: {pts}")
    return {"workload": f"config5: Llama-3-70B (K,N) qkv 8192x10240, o 8192x8192, gate_up 8192x57344, "
                        f"down 28672x8192; N split over {world} GPU(s); M in {list(TP_M)}",
            "collective": "NCCL all_gather_into_tensor of the output shards (shard-major, no reorder)" if world > 1 else "none",
            "parity": "gathered output == one-GPU output within normwise 1e-2 on sampled rows, every point, every rank",
            "points": pts}


MLP_M = (1, 32, 256, 4096)


def mlp70b_tp(world: int, rank: int, dev, ops, warm):
    """Config 5 strong scaling on the Llama-3-70B MLP block (H 8192, I 28672): gate_up split by
    output rows with SiLU * mul fused on each rank, down split by input columns, one NCCL
    all-reduce of the [M, H] output (llm_serving_engine_b200.parallel.TensorParallelInt8MLP).
    End to end per M (max over ranks), CUDA graph over rotated weight copies (each rank's
    weights stream from HBM), CUDA events.  Rank 0 also times the unsplit block on one GPU in
    the same run (the other ranks wait), so every run states its own speed-up over one GPU; the
    split output is checked against the unsplit one (normwise 1e-2)."""
    from llm_serving_engine_b200.int8_linear import Int8LlamaMLP
    from llm_serving_engine_b200.parallel import TensorParallelInt8MLP

    H, I = 8192, 28672
    gf = torch.Generator(device=dev).manual_seed(4242)  # identical full weights on every rank
    q = {k: torch.randint(-127, 128, shape, generator=gf, device=dev, dtype=torch.int8)
         for k, shape in (("g", (I, H)), ("u", (I, H)), ("d", (H, I)))}
    sc = {k: torch.empty(q[k].shape[0], device=dev).uniform_(1e-4, 5e-4, generator=gf) for k in q}
    per_rank_bytes = 3 * I * H // world
    copies = max(1, min(6, -(-3 * 126 * 2**20 // per_rank_bytes)))
    mlps = [TensorParallelInt8MLP.from_quantized(q["g"], sc["g"], q["u"], sc["u"], q["d"], sc["d"])]
    gr = torch.Generator(device=dev).manual_seed(99 + rank)
    for _ in range(copies - 1):  # further weights of the same shapes: only rotate the reads past L2
        r = {k: torch.randint(-127, 128, q[k].shape, generator=gr, device=dev, dtype=torch.int8) for k in q}
        mlps.append(TensorParallelInt8MLP.from_quantized(r["g"], sc["g"], r["u"], sc["u"], r["d"], sc["d"]))
        del r
    single = Int8LlamaMLP.from_quantized(torch.cat([q["g"], q["u"]]), torch.cat([sc["g"], sc["u"]]), q["d"], sc["d"], I) \
        if rank == 0 else None
    del q
    torch.cuda.empty_cache()
    pts = []
    ok_all = True
    for M in MLP_M:
        x = torch.randn(M, H, generator=gf, device=dev).to(torch.bfloat16)  # same x on every rank

        def run(x=x):
            for m in mlps:
                m(x)
        g = capture(run, warm)
        time_graph(g, 2)
        t = time_graph(g, 5) / len(mlps)
        del g
        t = max_over_ranks(t, world)
        y = mlps[0](x)
        t1, err = None, 0.0
        if rank == 0:
            def run1(x=x):
                for _ in range(3):
                    single(x)
            g1 = capture(run1, warm)
            time_graph(g1, 1)
            t1 = time_graph(g1, 3) / 3
            del g1
            ref = single(x).float()
            err = ((y.float() - ref).abs().max() / ref.abs().max().clamp_min(1e-30)).item()
        barrier(world)
        ok = max_over_ranks(0.0 if err <= 1e-2 else 1.0, world) == 0.0
        ok_all = ok_all and ok
        pt = {"M": M, "e2e_us": round(t * 1e3, 2), "TFLOPs": round(6.0 * M * H * I / t / 1e9, 1),
              "weight_GBps_per_gpu": round(per_rank_bytes / t / 1e6, 1), "parity_vs_one_gpu_ok": ok}
        if t1 is not None:
            pt["one_gpu_us"] = round(t1 * 1e3, 2)
            pt["speedup_vs_one_gpu"] = round(t1 / t, 3)
        pts.append(pt)
        del x, y
    del mlps, single
    torch.cuda.empty_cache()
    if not ok_all:
        raise RuntimeError(f"config5 MLP split: output differs from the one-GPU block: {pts}")
    return {"workload": f"config5: Llama-3-70B MLP block (H {H}, I {I}), gate_up rows and down columns split over "
                        f"{world} GPU(s), one NCCL all-reduce of the output; M in {list(MLP_M)}",
            "n_gpus": world, "collective": "NCCL all_reduce (sum) of the bf16 [M, H] output" if world > 1 else "none",
            "points": pts}


# --------------------------------------------------------------------------------------
def e2e_decode(dev, warm, hbm_peak, steps: int = 20):
    """Config 4: batched decode of a random-init Llama-3-8B-shaped model, 64 sequences at a
    1024-token context, one CUDA graph per step, int8 projections vs bf16 projections on the
    same weights (llm_serving_engine_b200.llama_decode).  tokens/s = 64 x steps / time."""
    from llm_serving_engine_b200.llama_decode import LLAMA3_8B, DecodeModel, decode_bytes_per_step

    B, ctx = 64, 1024
    base = DecodeModel(LLAMA3_8B, B, ctx, dev, seed=11, quantize=False, attention="paged")
    q8 = DecodeModel(LLAMA3_8B, B, ctx, dev, seed=11, quantize=True, weights=base.weights, kv=base.kv,
                     attention="paged")
    q8_sdpa = DecodeModel(LLAMA3_8B, B, ctx, dev, seed=11, quantize=True, weights=base.weights, attention="sdpa")
    q8_sdpa.proj = q8.proj  # same int8 modules, torch SDPA over a contiguous cache
    out = {"workload": "config4: Llama-3-8B shape (32 layers, hidden 4096, 32/8 heads, head_dim 128, MLP 14336, "
                       "vocab 128256), random init, 64 sequences, 1024-token context, greedy, CUDA graph per step; "
                       "attention: this package's paged decode-attention kernel over a block_size-16 pool in the "
                       "reference's layout; int8_sdpa: torch SDPA (cuDNN) over a contiguous cache",
           "unit": "tokens/s"}
    for name, m in (("int8", q8), ("int8_lm_head", q8), ("none", base), ("int8_sdpa", q8_sdpa)):
        q8.set_lm_head_int8(name == "int8_lm_head")
        g = capture(m.step, warm)
        time_graph(g, 3)
        ms = time_graph(g, steps)
        byts = decode_bytes_per_step(LLAMA3_8B, B, ctx, name != "none", int8_lm_head=name == "int8_lm_head")
        out[name] = {"tokens_per_s": round(B / (ms / 1e3), 1), "ms_per_step": round(ms, 4),
                     "bytes_per_step": byts, "GBps": round(byts / ms / 1e6, 1),
                     "frac_of_hbm": round(byts / ms / 1e6 / hbm_peak, 4)}
        del g
    out["int8_speedup"] = round(out["int8"]["tokens_per_s"] / out["none"]["tokens_per_s"], 3)
    out["int8_lm_head_speedup"] = round(out["int8_lm_head"]["tokens_per_s"] / out["none"]["tokens_per_s"], 3)
    q8.set_lm_head_int8(False)
    # the same model at small batches (the decode kernel's regime): int8 vs bf16 projections
    small = {}
    for b in (1, 16):
        bf = DecodeModel(LLAMA3_8B, b, ctx, dev, seed=11, quantize=False, weights=base.weights)
        i8 = DecodeModel(LLAMA3_8B, b, ctx, dev, seed=11, quantize=False, weights=base.weights, kv=bf.kv)
        i8.proj, i8.quantize = q8.proj, True  # the int8 modules built above
        row = {}
        for name, m in (("int8", i8), ("int8_lm_head", i8), ("none", bf)):
            i8.set_lm_head_int8(name == "int8_lm_head")
            g = capture(m.step, warm)
            time_graph(g, 3)
            ms = time_graph(g, steps)
            row[name] = {"tokens_per_s": round(b / (ms / 1e3), 1), "ms_per_step": round(ms, 4)}
            del g
        i8.set_lm_head_int8(False)
        row["int8_speedup"] = round(row["int8"]["tokens_per_s"] / row["none"]["tokens_per_s"], 3)
        row["int8_lm_head_speedup"] = round(row["int8_lm_head"]["tokens_per_s"] / row["none"]["tokens_per_s"], 3)
        small[f"batch{b}"] = row
        del bf, i8
    out["small_batch"] = small
    del base, q8, q8_sdpa
    torch.cuda.empty_cache()
    return out


def engine_decode(dev, hbm_peak: float, steps: int = 20, warmup: int = 5, batch: int = 64, context: int = 1024):
    """Config 4 through the reference engine itself (its install in baseline/_ref): the
    reference's `ModelRunner` with `use_custom_kernels` and `use_cuda_graphs`, decode graphs
    captured at bucket `batch` (`capture_decode_graphs`, `_self_check` included), a
    block_size-16 paged KV pool, `batch` greedy sequences prefilled to `context` tokens through
    `forward_fused`, then decode steps through `ModelRunner.forward` (graph replay with the
    engine's own host work: plan flattening, pinned H2D of the paging rows, one sampling sync
    per step).  tokens/s = batch x steps / wall time.

    Arms: `bf16_reference` (the stock engine: cuBLAS projections, its Triton paged attention),
    `bf16_lse` (bf16 projections with every binding that applies to them: `attend_paged` on
    this package's attention kernel, the RMSNorm kernel in the norm slots), `int8` (the
    `quantize="int8"` switch through `engine_hook.install()` with its defaults: int8
    projections, the same attention and norms, `write_kv_and_project_q` on the fused int8
    QKV output with the RoPE + K/V write kernel, and the residual adds in the o_proj and down
    epilogues) and `int8_no_rope` (the switch without those last two bindings: against
    `bf16_lse` it differs in the projections alone); and in fp16, the
    reference's default dtype, `fp16_reference` (the stock engine) and `fp16_int8` (the switch
    with its defaults).  The weights are a random-init Llama-3-8B (seeded, built on the
    GPU in place of `from_pretrained`: no checkpoint exists here); everything after the load is
    the engine's unmodified code."""
    import gc

    ref_dir = os.path.join(REPO, "baseline", "_ref")
    if os.path.isdir(ref_dir) and ref_dir not in sys.path:
        sys.path.insert(0, ref_dir)
    try:
        import llm_serving_engine.model.model_runner as mr
        from llm_serving_engine.config import ModelConfig
        from llm_serving_engine.model.sampling import SamplingParams
        from llm_serving_engine.observability.metrics import RequestMetrics
        from llm_serving_engine.scheduling.allocator import BlockAllocator
        from llm_serving_engine.scheduling.batch_plan import BatchEntry, BatchPlan
        from llm_serving_engine.scheduling.sequence import Sequence
    except Exception as e:  # noqa: BLE001 - the reference is optional here
        return {"unavailable": f"the reference engine is not importable from baseline/_ref: {e}"}
    from transformers import LlamaConfig, LlamaForCausalLM

    from llm_serving_engine_b200 import engine_hook
    from llm_serving_engine_b200.llama_decode import LLAMA3_8B, decode_bytes_per_step

    cfg = LlamaConfig(vocab_size=128256, hidden_size=4096, intermediate_size=14336, num_hidden_layers=32,
                      num_attention_heads=32, num_key_value_heads=8, max_position_embeddings=8192,
                      rope_theta=500000.0, rms_norm_eps=1e-5, bos_token_id=None, eos_token_id=None,
                      pad_token_id=None, tie_word_embeddings=False)

    class _SyntheticLoader:
        @staticmethod
        def from_pretrained(path, dtype=None, **kwargs):
            torch.manual_seed(0)
            with torch.device(dev):
                model = LlamaForCausalLM(cfg)
            return model.to(dtype)

    bs = 16
    nblocks = batch * (-(-(context + warmup + steps + 1) // bs)) + 8
    out = {"workload": f"config4 through the reference ModelRunner: Llama-3-8B shape, random init, {batch} sequences "
                       f"prefilled to {context} tokens, greedy, decode graphs at bucket {batch}, block_size {bs}",
           "unit": "tokens/s", "timing": "wall clock over the steps (each step ends in the engine's sampling sync)"}
    original_loader = mr.AutoModelForCausalLM
    mr.AutoModelForCausalLM = _SyntheticLoader
    try:
        for arm in ("bf16_reference", "bf16_lse", "int8_no_rope", "int8", "fp16_reference", "fp16_int8"):
            quantize = "int8" if "int8" in arm else "none"
            if quantize == "int8":
                engine_hook.install(rope=arm != "int8_no_rope", residuals=arm != "int8_no_rope")
            try:
                runner = mr.ModelRunner(ModelConfig(model_name_or_path="synthetic-llama-3-8b", device=str(dev),
                                                    dtype="float16" if arm.startswith("fp16") else "bfloat16",
                                                    quantize=quantize))
            finally:
                engine_hook.uninstall()
            if arm == "bf16_lse":
                engine_hook.bind_paged_attention(runner)
                engine_hook.bind_rms_norms(runner)
            runner.allocate_kv_pool(nblocks, bs)
            runner.capture_decode_graphs([batch])
            graphs_kept = batch in runner._decode_graphs.graphs
            alloc = BlockAllocator(nblocks, bs)
            gen = torch.Generator().manual_seed(5)
            seqs = [Sequence(seq_id=i, prompt_tokens=torch.randint(1, 128000, (context,), generator=gen).tolist(),
                             sampling_params=SamplingParams(temperature=0.0, max_tokens=1 << 20),
                             metrics=RequestMetrics(enqueue_time=0.0)) for i in range(batch)]
            by_id = {s.seq_id: s for s in seqs}
            for c in range(0, batch, 8):  # prefill, 8 prompts per iteration (the scheduler's bookkeeping)
                entries = []
                for s in seqs[c:c + 8]:
                    assert alloc.allocate(s, s.num_tokens)
                    s.prefill_progress += s.num_tokens
                    s.status = "DECODING"
                    entries.append(BatchEntry(s.seq_id, s.num_tokens, is_prefill_chunk=True))
                for sid, tok, _ in runner.forward(BatchPlan(entries=entries), by_id):
                    by_id[sid].generated_tokens.append(tok)
                    assert alloc.allocate(by_id[sid], 1)
            eager = {"n": 0}
            fused = runner.forward_fused

            def counting_fused(*a, **k):
                eager["n"] += 1
                return fused(*a, **k)

            runner.forward_fused = counting_fused

            def step():
                plan = BatchPlan(entries=[BatchEntry(s.seq_id, 1, is_prefill_chunk=False) for s in seqs])
                for sid, tok, _ in runner.forward(plan, by_id):
                    by_id[sid].generated_tokens.append(tok)
                    assert alloc.allocate(by_id[sid], 1)

            for _ in range(warmup):
                step()
            torch.cuda.synchronize()
            eager["n"] = 0
            t0 = time.perf_counter()
            for _ in range(steps):
                step()
            torch.cuda.synchronize()
            sec = time.perf_counter() - t0
            # the step's HBM bound (weights, K/V at the mean context of the timed steps, lm_head)
            byts = decode_bytes_per_step(LLAMA3_8B, batch, context + warmup + steps // 2, quantize == "int8")
            out[arm] = {"tokens_per_s": round(batch * steps / sec, 1), "ms_per_step": round(sec / steps * 1e3, 4),
                        "bytes_per_step": byts, "GBps": round(byts * steps / sec / 1e9, 1),
                        "frac_of_hbm": round(byts * steps / sec / 1e9 / hbm_peak, 4),
                        "decode_graph_kept": graphs_kept, "eager_steps_in_timed_region": eager["n"],
                        "context_at_end": seqs[0].num_tokens}
            del runner, seqs, by_id, alloc
            gc.collect()
            torch.cuda.empty_cache()
    finally:
        mr.AutoModelForCausalLM = original_loader
    out["int8_speedup_vs_bf16_reference"] = round(out["int8"]["tokens_per_s"] / out["bf16_reference"]["tokens_per_s"], 3)
    out["int8_speedup_vs_bf16_lse"] = round(out["int8"]["tokens_per_s"] / out["bf16_lse"]["tokens_per_s"], 3)
    out["int8_no_rope_speedup_vs_bf16_lse"] = round(
        out["int8_no_rope"]["tokens_per_s"] / out["bf16_lse"]["tokens_per_s"], 3)
    out["fp16_int8_speedup_vs_fp16_reference"] = round(
        out["fp16_int8"]["tokens_per_s"] / out["fp16_reference"]["tokens_per_s"], 3)
    return out


def fused_gate_up(weights, dev, warm, ops, hbm_peak):
    """The MLP's first half, silu(x Wg^T) * (x Wu^T), over every layer's gate_up weight: one
    fused launch (lse_int8_gate_up_silu_packed[_ws]: the decode kernel for M <= 16, the
    tcgen05 kernel with SiLU * mul in its epilogue above; gate and up rows interleaved in
    8-row blocks) vs the int8 gate_up projection followed by torch's SiLU * mul, at decode
    (1, 4, 16, 64) and prefill (512, 2048) token counts.  The uniform random weights stand
    for an interleaved [gate; up] as they are."""
    K, N2 = LLAMA3_8B_SHAPES["gate_up"]
    inter = N2 // 2
    gx = torch.Generator(device=dev).manual_seed(17)
    out = {"workload": f"Llama-3-8B gate_up K={K}, I={inter}, {len(weights)} layers' weights per graph", "points": []}
    for M in (1, 4, 16, 64, 512, 2048):
        x = torch.randn(M, K, generator=gx, device=dev).to(torch.bfloat16)
        h = torch.empty(M, inter, device=dev, dtype=torch.bfloat16)
        gu = torch.empty(M, N2, device=dev, dtype=torch.bfloat16)

        def fused(x=x, h=h):
            for layer in weights:
                wp, s = layer["gate_up"]
                ops.int8_gate_up_silu_packed(x, wp, s, inter, K, out=h)

        def unfused(x=x, gu=gu, h=h):
            for layer in weights:
                wp, s = layer["gate_up"]
                ops.int8_linear_packed(x, wp, s, N2, K, out=gu)
                torch.mul(F.silu(gu[:, :inter]), gu[:, inter:], out=h)
        pt = {"M": M}
        for name, fn in (("fused", fused), ("unfused", unfused)):
            g = capture(fn, warm)
            time_graph(g, 2)
            us = time_graph(g, 10) / len(weights) * 1e3
            pt[name + "_us"] = round(us, 3)
            del g
        b = linear_bytes(M, K, N2) - M * N2 * 2 + M * inter * 2
        pt["fused_GBps"] = round(b / pt["fused_us"] / 1e3, 1)
        pt["fused_frac_of_hbm"] = round(b / pt["fused_us"] / 1e3 / hbm_peak, 4)
        pt["fused_TFLOPs"] = round(2 * M * K * N2 / pt["fused_us"] / 1e6, 1)
        pt["speedup"] = round(pt["unfused_us"] / pt["fused_us"], 3)
        out["points"].append(pt)
    return out


def fused_residual(weights, dev, warm, ops):
    """The decoder's residual add fused into the projection epilogue (o_proj and down, whose
    outputs are added to the residual stream): `int8_linear_packed(..., residual=h)` vs the
    projection followed by torch's add, at M in 1, 4, 16, 64 over every layer's weight."""
    gx = torch.Generator(device=dev).manual_seed(19)
    out = {"workload": f"Llama-3-8B o (4096x4096) and down (14336x4096), {len(weights)} layers' weights per graph",
           "points": []}
    for name in ("o", "down"):
        K, N = LLAMA3_8B_SHAPES[name]
        for M in DECODE_M:
            x = torch.randn(M, K, generator=gx, device=dev).to(torch.bfloat16)
            h = torch.randn(M, N, generator=gx, device=dev).to(torch.bfloat16)
            y = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
            h2 = torch.empty_like(h)

            def fused(x=x, h=h, h2=h2, name=name, N=N, K=K):
                for layer in weights:
                    wp, s = layer[name]
                    ops.int8_linear_packed(x, wp, s, N, K, out=h2, residual=h)

            def unfused(x=x, h=h, y=y, h2=h2, name=name, N=N, K=K):
                for layer in weights:
                    wp, s = layer[name]
                    ops.int8_linear_packed(x, wp, s, N, K, out=y)
                    torch.add(h, y, out=h2)
            pt = {"shape": name, "M": M}
            for tag, fn in (("fused", fused), ("unfused", unfused)):
                g = capture(fn, warm)
                time_graph(g, 2)
                pt[tag + "_us"] = round(time_graph(g, 10) / len(weights) * 1e3, 3)
                del g
            pt["speedup"] = round(pt["unfused_us"] / pt["fused_us"], 3)
            out["points"].append(pt)
    return out


def decode_attention(dev, warm, ops, hbm_peak):
    """The paged decode-attention kernel alone: Llama-3-8B attention shape (32 query / 8 KV
    heads, head_dim 128), 1025 positions per sequence in a block_size-16 pool with a shuffled
    block table, one pool per layer for 32 layers in a CUDA graph (the K/V stream exceeds L2
    for E >= 16).  GB/s = K and V bytes read / time."""
    H, H_kv, D, bs, ctx, layers = 32, 8, 128, 16, 1025, 32
    out = {"workload": f"H={H}, H_kv={H_kv}, D={D}, block_size={bs}, context {ctx}, {layers} layers' pools per graph",
           "points": []}
    g = torch.Generator(device=dev).manual_seed(23)
    for E in (1, 16, 64):
        nbps = -(-ctx // bs)
        nb = E * nbps + 1
        bt = torch.randperm(nb, device=dev, generator=g)[: E * nbps].view(E, nbps).to(torch.int32)
        cl = torch.full((E,), ctx, dtype=torch.int32, device=dev)
        pools = [(torch.randn(nb, bs, H_kv, D, device=dev, generator=g).to(torch.bfloat16),
                  torch.randn(nb, bs, H_kv, D, device=dev, generator=g).to(torch.bfloat16)) for _ in range(layers)]
        q = torch.randn(E, H, D, device=dev, generator=g).to(torch.bfloat16)
        o = torch.empty_like(q)

        def run(q=q, o=o, pools=pools, bt=bt, cl=cl):
            for kp, vp in pools:
                ops.paged_decode_attention(q, kp, vp, bt, cl, ctx, out=o)
        gr = capture(run, warm)
        time_graph(gr, 2)
        us = time_graph(gr, 10) / layers * 1e3
        byts = E * ctx * H_kv * D * 2 * 2
        out["points"].append({"E": E, "us": round(us, 3), "GBps": round(byts / us / 1e3, 1),
                              "frac_of_hbm": round(byts / us / 1e3 / hbm_peak, 4)})
        del gr, pools
        torch.cuda.empty_cache()
    return out


def prefill_attention(dev, warm, ops):
    """The multi-token paged-attention kernel (prefill chunks) beside the reference's Triton
    `paged_attention_forward` when its install is importable: Llama-3-8B attention shape,
    bf16, one chunk of q_len tokens after a cached prefix per entry.  TFLOP/s counts the
    causal work (4 * D flops per query-key pair seen)."""
    ref_dir = os.path.join(REPO, "baseline", "_ref")
    if os.path.isdir(ref_dir) and ref_dir not in sys.path:
        sys.path.insert(0, ref_dir)
    try:
        from llm_serving_engine.kernels.flash_attention import paged_attention_forward as ref_fwd
    except Exception:  # the reference is not installed: our kernel alone
        ref_fwd = None
    H, H_kv, D, bs = 32, 8, 128, 16
    out = {"workload": f"H={H}, H_kv={H_kv}, D={D}, block_size={bs}, bf16", "points": []}
    g = torch.Generator(device=dev).manual_seed(29)
    for E, qlen, prefix in ((1, 2048, 0), (4, 512, 1024), (16, 128, 896)):
        ctx = prefix + qlen
        nbps = -(-ctx // bs)
        nb = E * nbps + 1
        bt = torch.randperm(nb, device=dev, generator=g)[: E * nbps].view(E, nbps).to(torch.int32)
        i32 = lambda v: torch.tensor(v, dtype=torch.int32, device=dev)
        cl, off = i32([ctx] * E), i32([prefix] * E)
        qs, ql = i32([e * qlen for e in range(E)]), i32([qlen] * E)
        kp = torch.randn(nb, bs, H_kv, D, device=dev, generator=g).to(torch.bfloat16)
        vp = torch.randn(nb, bs, H_kv, D, device=dev, generator=g).to(torch.bfloat16)
        q = torch.randn(H, E * qlen, D, device=dev, generator=g).to(torch.bfloat16)
        pairs = E * H * sum(min(ctx, prefix + i + 1) for i in range(qlen))
        flops = 4.0 * D * pairs
        pt = {"E": E, "q_len": qlen, "prefix": prefix}
        for name, fn in (("ours", lambda: ops.paged_attention(q, kp, vp, bt, cl, off, qs, ql, bs, qlen)),
                         ("reference_triton", (lambda: ref_fwd(q, kp, vp, bt, cl, off, qs, ql, bs, qlen)) if ref_fwd else None)):
            if fn is None:
                continue
            def run(fn=fn):
                for _ in range(8):
                    fn()
            gr = capture(run, warm)
            time_graph(gr, 2)
            us = time_graph(gr, 10) / 8 * 1e3
            pt[f"{name}_us"] = round(us, 2)
            pt[f"{name}_TFLOPs"] = round(flops / us / 1e6, 1)
            del gr
        if "reference_triton_us" in pt:
            pt["speedup"] = round(pt["reference_triton_us"] / pt["ours_us"], 3)
        out["points"].append(pt)
        del kp, vp, q
        torch.cuda.empty_cache()
    return out


def host_overhead(dev, ops):
    """Host time per projection call at M = 16 (Llama-3-8B o_proj shape), no synchronization in
    the loop: the ctypes path (`ops.int8_linear_packed`), the dispatcher operator
    (`torch.ops.lse.int8_linear`, what the int8 modules call) and torch's bf16 `F.linear`
    (cuBLAS) for comparison, each with its launch count per call."""
    K, N, M, calls = 4096, 4096, 16, 2000
    x = torch.randn(M, K, device=dev).to(torch.bfloat16)
    w = ops.pack_weight(torch.randint(-127, 128, (N, K), device=dev, dtype=torch.int8))
    s = torch.rand(N, device=dev) * 1e-3
    wb = torch.randn(N, K, device=dev).to(torch.bfloat16)
    lse = ops.torch_ops()
    cases = {"ctypes_ops_int8_linear_packed": lambda: ops.int8_linear_packed(x, w, s, N, K),
             "torch_ops_lse_int8_linear": lambda: lse.int8_linear(x, w, s, N, K),
             "torch_F_linear_bf16": lambda: torch.nn.functional.linear(x, wb)}
    out = {"workload": f"M={M}, K={K}, N={N}, {calls} calls, host wall time per call (GPU queue not drained)",
           "launches_per_call": {"ctypes_ops_int8_linear_packed": 1, "torch_ops_lse_int8_linear": 1,
                                 "torch_F_linear_bf16": 1}}
    for name, fn in cases.items():
        for _ in range(50):
            fn()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(calls):
            fn()
        out[name + "_us"] = round((time.perf_counter() - t0) / calls * 1e6, 2)
        torch.cuda.synchronize()
    return out


def bf16_cublas_points(layers: int, dev, warm, xs):
    """Same-box comparison: torch F.linear (cuBLAS) with bf16 weights of the same shapes at
    every decode-sweep point, `layers` distinct weights per graph (the reference's
    quantize="none" projections).  Per point: us per launch and bf16 weight GB/s."""
    g = torch.Generator(device=dev).manual_seed(29)
    wts = {name: [torch.randn(N, K, generator=g, device=dev).to(torch.bfloat16) for _ in range(layers)]
           for name, (K, N) in LLAMA3_8B_SHAPES.items()}
    out = []
    for M in DECODE_M:
        for name in SHAPE_ORDER:
            K, N = LLAMA3_8B_SHAPES[name]
            y = torch.empty(M, N, device=dev, dtype=torch.bfloat16)

            def one(x=xs[(M, name)], y=y, ws=wts[name]):
                for w in ws:
                    torch.matmul(x, w.t(), out=y)
            gr = capture(one, warm)
            time_graph(gr, 2)
            us = time_graph(gr, 10) / layers * 1e3
            out.append({"M": M, "shape": name, "us": round(us, 3),
                        "GBps": round((2 * N * K + 2 * M * K + 2 * M * N) / us / 1e3, 1)})
            del gr
    del wts
    torch.cuda.empty_cache()
    return out


# --------------------------------------------------------------------------------------
def cpu_reference_sample(seconds: float):
    """The reference's CPU path (float32 nn.Linear on the dequantized weight, all host
    threads) over one layer of the decode sweep, repeated for ~`seconds`."""
    from llm_serving_engine_b200.inputs import make_inputs
    from oracle.cpu_path import ReferenceCpuLinear, cpu_model, host_threads

    threads = host_threads()
    mods, xs, nbytes = {}, {}, 0
    for name in SHAPE_ORDER:
        K, N = LLAMA3_8B_SHAPES[name]
        x, w, s = make_inputs(max(DECODE_M), K, N, seed=0)
        mods[name] = ReferenceCpuLinear(w, s)
        for M in DECODE_M:
            xs[(M, name)] = x[:M].float().contiguous()
            nbytes += linear_bytes(M, K, N)
    for M in DECODE_M:  # warm-up pass
        for name in SHAPE_ORDER:
            mods[name](xs[(M, name)])
    passes, t0 = 0, time.perf_counter()
    while True:
        for M in DECODE_M:
            for name in SHAPE_ORDER:
                mods[name](xs[(M, name)])
        passes += 1
        el = time.perf_counter() - t0
        if el >= seconds or passes >= 1000:
            break
    gbs = nbytes * passes / el / 1e9
    return {
        "value": round(gbs, 3), "unit": UNIT, "cores": threads, "kind": "port",
        "sample": f"{passes} passes of the 16 decode-sweep points (1 layer of weights), float32 torch "
                  f"F.linear on dequantized weights, {el:.1f} s, CPU {cpu_model()}",
    }, el / passes


def run_reference(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    from llm_serving_engine_b200.inputs import make_inputs
    from oracle.cpu_path import ReferenceCpuLinear, cpu_model, host_threads

    threads = host_threads()
    mods, xs, nbytes = {}, {}, 0
    for name in SHAPE_ORDER:
        K, N = LLAMA3_8B_SHAPES[name]
        x, w, s = make_inputs(max(DECODE_M), K, N, seed=0)
        mods[name] = ReferenceCpuLinear(w, s)
        for M in DECODE_M:
            xs[(M, name)] = x[:M].float().contiguous()
            nbytes += linear_bytes(M, K, N)

    def step():
        for M in DECODE_M:
            for name in SHAPE_ORDER:
                mods[name](xs[(M, name)])

    for _ in range(max(args.warmup, 1)):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    el = time.perf_counter() - t0
    gbs = nbytes * args.steps / el / 1e9
    sample = (f"each step: the 16 decode-sweep points over 1 layer of weights (the GPU arm's step runs "
              f"32 layers), float32 torch F.linear on dequantized weights (the reference's CPU nn.Linear "
              f"path; it has no int8 kernel), CPU {cpu_model()}")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(el / args.steps * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "config2 decode sweep (M in 1,4,16,64 x Llama-3-8B qkv/o/gate_up/down), 1-layer sample on CPU"},
        "cpu_baseline": {"value": round(gbs, 3), "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": round(gbs, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# --------------------------------------------------------------------------------------
def main():
    args = parse_args()
    if args.impl == "reference":
        return run_reference(args)
    world, rank, local = setup_dist(args)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)

    from llm_serving_engine_b200 import ops

    hbm_peak, bf16_peak, bf16_sustained, peak_src = peaks()
    layers = args.layers
    weights = make_weights(layers, dev, seed=1000 + rank, ops=ops)
    gx = torch.Generator(device=dev).manual_seed(7 + rank)
    xs, ys = {}, {}
    for M in DECODE_M:
        for name in SHAPE_ORDER:
            K, N = LLAMA3_8B_SHAPES[name]
            xs[(M, name)] = torch.randn(M, K, generator=gx, device=dev).to(torch.bfloat16)
            ys[(M, name)] = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
    step_bytes = sum(linear_bytes(M, *LLAMA3_8B_SHAPES[n]) for M in DECODE_M for n in SHAPE_ORDER) * layers
    launches_per_step = len(DECODE_M) * len(SHAPE_ORDER) * layers

    warm = torch.cuda.Stream(device=dev)
    step = decode_step_fn(weights, xs, ys, ops)
    graph = capture(step, warm)

    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(args.steps):
            graph.replay()
        end.record()
        torch.cuda.synchronize()
    barrier(world)
    ms = start.elapsed_time(end)
    ms_max = max_over_ranks(ms, world)
    value = step_bytes * args.steps * world / (ms_max / 1e3) / 1e9
    ms_per_step = ms_max / args.steps

    # ---- per-point breakdown: one graph per (M, shape) over all layers -----------------
    # The auto policy of lse_int8_linear_packed: the warp-MMA skinny kernel for M <= 16, the
    # tcgen05 kernel above.
    points = []
    per_kernel = {"skinny_i8_kernel": [0.0, 0.0, 0], "tc_i8_kernel": [0.0, 0.0, 0]}  # bytes, ms, launches
    for M in DECODE_M:
        for name in SHAPE_ORDER:
            K, N = LLAMA3_8B_SHAPES[name]

            def one(M=M, name=name):
                for layer in weights:
                    wp, s = layer[name]
                    linear_call(ops, xs[(M, name)], wp, s, ys[(M, name)], name)
            g1 = capture(one, warm)
            time_graph(g1, 2)
            per_launch_ms = time_graph(g1, 10) / layers
            b = linear_bytes(M, K, N)
            kern = "skinny_i8_kernel" if M <= 16 else "tc_i8_kernel"
            per_kernel[kern][0] += b
            per_kernel[kern][1] += per_launch_ms
            per_kernel[kern][2] += 1
            points.append({"M": M, "shape": name, "K": K, "N": N, "us": round(per_launch_ms * 1e3, 3),
                           "GBps": round(b / per_launch_ms / 1e6, 1), "kernel": kern})
            del g1
    traffic = committed_traffic()

    def roof(kern):
        b, ms, n = per_kernel[kern]
        achieved = b / ms / 1e6
        tr = traffic.get(kern)
        return {
            "kernel": kern, "bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
            "frac": round(achieved / hbm_peak, 4),
            "peak_source": ("measured: MEASURED_PEAKS.json hbm_gbs (copy, read+write)" if peak_src == "measured"
                            else "fallback 6650 GB/s"),
            "frac_of_8TBps": round(achieved / 8000.0, 4),
            "algorithmic_bytes_per_launch": round(b / n),
            # DRAM bytes per launch from one ncu capture of a named case (profiles/traffic.json),
            # beside that case's own algorithmic bytes: their ratio is the re-read factor
            "traffic": tr.get("dram_bytes_per_launch") if tr else None,
            "traffic_case": tr.get("case") if tr else None,
            "traffic_case_algorithmic_bytes": tr.get("algorithmic_bytes_per_launch") if tr else None,
            "traffic_ratio": (round(tr["dram_bytes_per_launch"] / tr["algorithmic_bytes_per_launch"], 4)
                              if tr and tr.get("algorithmic_bytes_per_launch") else None),
        }
    # dominant kernel = the one with the larger share of the step's time
    step_share = {k: v[1] for k, v in per_kernel.items()}
    dominant = max(step_share, key=step_share.get)
    roofline = roof(dominant)
    roofline["share_of_step"] = round(step_share[dominant] / sum(step_share.values()), 3)
    roofline_other = roof(min(step_share, key=step_share.get))

    # ---- prefill (config 3) ------------------------------------------------------------
    prefill = None
    if not args.no_prefill:
        pre_pts, fl_tot, ms_tot = [], 0.0, 0.0
        layer0 = weights[0]
        for M in PREFILL_M:
            for name in SHAPE_ORDER:
                K, N = LLAMA3_8B_SHAPES[name]
                xp = torch.randn(M, K, generator=gx, device=dev).to(torch.bfloat16)
                yp = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
                wp, s = layer0[name]

                def one(xp=xp, yp=yp, wp=wp, s=s, name=name):
                    linear_call(ops, xp, wp, s, yp, name)
                g1 = capture(one, warm)
                time_graph(g1, 2)
                t = time_graph(g1, 10)
                fl = linear_flops(M, K, N)
                fl_tot += fl
                ms_tot += t
                pre_pts.append({"M": M, "shape": name, "us": round(t * 1e3, 2), "TFLOPs": round(fl / t / 1e9, 1)})
                del g1, xp, yp
        tf = fl_tot / ms_tot / 1e9
        prefill = {"value": round(tf, 1), "unit": "TFLOP/s", "workload": "config3: M in 512,2048,8192 x 4 shapes",
                   "roofline": {"bound": "tensor", "achieved": round(tf, 1), "peak": bf16_peak, "unit": "TFLOP/s",
                                "frac": round(tf / bf16_peak, 4), "frac_of_2250": round(tf / 2250.0, 4),
                                "peak_source": peak_src + " bf16_tflops (burst)"},
                   "points": pre_pts}

    fused_mlp = fused_gate_up(weights, dev, warm, ops, hbm_peak)
    fused_res = fused_residual(weights, dev, warm, ops)
    attn = decode_attention(dev, warm, ops, hbm_peak)
    pattn = prefill_attention(dev, warm, ops)
    host = host_overhead(dev, ops)
    cublas = bf16_cublas_points(layers, dev, warm, xs)
    tp70b = None if args.no_70b else tp70b_sweep(world, rank, dev, ops, warm)
    mlp70b = None if args.no_70b else mlp70b_tp(world, rank, dev, ops, warm)
    decode4 = e2e_decode(dev, warm, hbm_peak) if (world == 1 and not args.no_e2e_decode) else None
    engine4 = engine_decode(dev, hbm_peak) if (world == 1 and not args.no_engine_decode) else None

    # ---- e2e: pinned host activations in, graph replay, outputs back, every step -------
    host_x = {k: v.cpu().pin_memory() for k, v in xs.items()}
    host_y = {k: torch.empty(v.shape, dtype=v.dtype).pin_memory() for k, v in ys.items()}
    h2d = sum(v.numel() * v.element_size() for v in host_x.values())
    d2h = sum(v.numel() * v.element_size() for v in host_y.values())
    e2e_steps = max(1, min(args.steps, 50))
    torch.cuda.synchronize()
    barrier(world)
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        for k, v in host_x.items():
            xs[k].copy_(v, non_blocking=True)
        graph.replay()
        for k, v in ys.items():
            host_y[k].copy_(v, non_blocking=True)
        torch.cuda.current_stream().synchronize()
    e2e_s = time.perf_counter() - t0
    e2e_s = max_over_ranks(e2e_s, world)
    e2e_val = step_bytes * e2e_steps * world / e2e_s / 1e9

    cpu_base = None
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        cpu_base, _ = cpu_reference_sample(args.cpu_seconds)

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16 x int8 (fp32 accumulate)",
            "data": "synthetic (seeded: x~N(0,1) bf16, W uniform int8 [-127,127], s uniform [1e-4,5e-4])",
            "config": {
                "workload": "config2 decode sweep: M in 1,4,16,64 x Llama-3-8B (K,N) qkv 4096x6144, o 4096x4096, "
                            "gate_up 4096x28672, down 14336x4096",
                "layers": layers, "launches_per_step": launches_per_step,
                "bytes_per_step": step_bytes, "l2": "inputs larger than L2 (6.98 GB of distinct int8 weights per M pass)",
                "graph": "one CUDA graph per step (decode-graph replay)",
                "parallelism": f"column stripes x{world}, no collective" if world > 1 else "single GPU",
            },
            "roofline": roofline,
            "roofline_other_kernel": roofline_other,
            "gpu_launches": launches_per_step * args.steps,
            "e2e": {"value": round(e2e_val, 1), "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "steps": e2e_steps, "how": "pinned host x -> device, graph replay, y -> pinned host, sync; wall clock"},
            "clocks": clk.summary(),
            "points": points,
        }
        if prefill:
            line["prefill"] = prefill
        line["fused_gate_up_silu"] = fused_mlp
        line["fused_residual"] = fused_res
        line["decode_attention"] = attn
        line["prefill_attention"] = pattn
        line["host_overhead"] = host
        line["bf16_cublas_points"] = cublas
        line["int8_speedup_vs_bf16_cublas"] = {f"M{p['M']}_{p['shape']}": round(c["us"] / p["us"], 3)
                                               for p, c in zip(points, cublas)}
        if tp70b:
            line["config5_70b_column_split"] = tp70b
        if mlp70b:
            line["config5_mlp_strong_scaling"] = mlp70b
        if decode4:
            line["config4_e2e_decode"] = decode4
        if engine4:
            line["config4_engine_decode"] = engine4
        if cpu_base:
            line["cpu_baseline"] = cpu_base
        print(json.dumps(line), flush=True)

    del graph
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
