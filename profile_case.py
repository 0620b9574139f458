"""Launch one int8-linear shape a few times: the small, self-contained workload the ncu
captures in profiles/ are taken on.

    python profile_case.py --M 16 --shape gate_up --algo tcgen05 --launches 4
    python profile_case.py --M 64 --gate-up-silu --launches 6
    python profile_case.py --decode-step 64 --launches 2      (a whole Llama-3-8B decode step)
    python profile_case.py --prefill-attention 1 --launches 4  (multi-token paged attention)

Weights (in the packed layout the module stores) are rotated over enough distinct copies that each launch reads its weight from
HBM, not from L2 (126 MB); the device footprint stays at a few GB.  Prints the CUDA-event
time per launch of back-to-back launches captured in one CUDA graph (not meaningful under a
profiler).  The graph is replayed twice: a capture of `--launches N` with ncu `-s N -c 1`
profiles the first launch of the second replay.
"""

from __future__ import annotations

import argparse

import torch

from llm_serving_engine_b200 import ops
from llm_serving_engine_b200.inputs import LLAMA3_8B_SHAPES, LLAMA3_70B_SHAPES, linear_bytes, linear_flops

ALGOS = {"auto": ops.ALGO_AUTO, "gemv": ops.ALGO_GEMV, "tcgen05": ops.ALGO_TCGEN05, "skinny": ops.ALGO_SKINNY}


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--M", type=int, default=16)
    ap.add_argument("--shape", default="gate_up")
    ap.add_argument("--model", choices=("8b", "70b"), default="8b")
    ap.add_argument("--algo", choices=list(ALGOS), default="auto")
    ap.add_argument("--launches", type=int, default=4)
    ap.add_argument("--rowmajor", action="store_true", help="row-major W instead of the packed layout")
    ap.add_argument("--gate-up-silu", action="store_true",
                    help="the fused gate_up + SiLU*mul (ops.int8_gate_up_silu_packed) on the gate_up shape")
    ap.add_argument("--attention", type=int, default=0, metavar="E",
                    help="profile the paged decode attention instead: E sequences of 1025 positions, "
                         "Llama-3-8B attention shape, three layers' pools in rotation")
    ap.add_argument("--decode-step", type=int, default=0, metavar="B",
                    help="time `--launches` CUDA-graph replays of one int8 decode step of a random-init "
                         "Llama-3-8B at B sequences x 1024 cached positions (llama_decode.DecodeModel), "
                         "inside an NVTX range 'step'")
    ap.add_argument("--prefill-attention", type=int, default=0, metavar="E",
                    help="profile the multi-token paged attention instead: E entries with a 2048 / E token "
                         "chunk each, Llama-3-8B attention shape")
    args = ap.parse_args(argv)
    if args.attention:
        return attention_case(args.attention, args.launches)
    if args.decode_step:
        return decode_step_case(args.decode_step, args.launches)
    if args.prefill_attention:
        return prefill_attention_case(args.prefill_attention, args.launches)
    if args.gate_up_silu:
        args.shape = "gate_up"
    K, N = (LLAMA3_8B_SHAPES if args.model == "8b" else LLAMA3_70B_SHAPES)[args.shape]
    copies = max(2, -(-3 * 128 * 2**20 // (N * K)))  # > 3x L2 of weights in rotation
    g = torch.Generator(device="cuda").manual_seed(0)
    ws = [torch.randint(-127, 128, (N, K), generator=g, device="cuda", dtype=torch.int8) for _ in range(copies)]
    if not args.rowmajor:
        ws = [ops.pack_weight(w) for w in ws]

    def call(w):
        if args.gate_up_silu:
            ops.int8_gate_up_silu_packed(x, w, s, N // 2, K, out=h)
        elif args.rowmajor:
            ops.int8_linear(x, w, s, out=y, algo=algo)
        else:
            ops.int8_linear_packed(x, w, s, N, K, out=y, algo=algo)
    s = torch.empty(N, device="cuda").uniform_(1e-4, 5e-4, generator=g)
    x = torch.randn(args.M, K, generator=g, device="cuda").to(torch.bfloat16)
    y = torch.empty(args.M, N, device="cuda", dtype=torch.bfloat16)
    h = torch.empty(args.M, N // 2, device="cuda", dtype=torch.bfloat16)
    algo = ALGOS[args.algo]
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        call(ws[0])  # first call on the capture stream creates its workspace
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        for i in range(args.launches):
            call(ws[i % copies])
    graph.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    graph.replay()
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / args.launches
    what = "fused gate_up+SiLU*mul" if args.gate_up_silu else f"algo={args.algo} {'row-major' if args.rowmajor else 'packed'}"
    print(f"M={args.M} {args.model}:{args.shape} K={K} N={N} {what}: {ms * 1e3:.2f} us/launch "
          f"({linear_bytes(args.M, K, N) / ms / 1e6:.0f} GB/s, {linear_flops(args.M, K, N) / ms / 1e9:.1f} TFLOP/s, "
          f"CUDA-graph launches)")
    assert ops.device_status() == 0


def attention_case(E: int, launches: int) -> None:
    """`launches` paged decode-attention calls (32 query / 8 KV heads, head_dim 128, block_size
    16, 1025 positions, shuffled block table) over three layers' pools, in one CUDA graph."""
    H, H_kv, D, bs, ctx = 32, 8, 128, 16, 1025
    g = torch.Generator(device="cuda").manual_seed(0)
    nbps = -(-ctx // bs)
    nb = E * nbps + 1
    bt = torch.randperm(nb, device="cuda", generator=g)[: E * nbps].view(E, nbps).to(torch.int32)
    cl = torch.full((E,), ctx, dtype=torch.int32, device="cuda")
    pools = [(torch.randn(nb, bs, H_kv, D, device="cuda", generator=g).to(torch.bfloat16),
              torch.randn(nb, bs, H_kv, D, device="cuda", generator=g).to(torch.bfloat16)) for _ in range(3)]
    q = torch.randn(E, H, D, device="cuda", generator=g).to(torch.bfloat16)
    o = torch.empty_like(q)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        ops.paged_decode_attention(q, *pools[0], bt, cl, ctx, out=o)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        for i in range(launches):
            ops.paged_decode_attention(q, *pools[i % 3], bt, cl, ctx, out=o)
    graph.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    graph.replay()
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / launches
    byts = E * ctx * H_kv * D * 2 * 2
    print(f"paged decode attention E={E} ctx={ctx}: {ms * 1e3:.2f} us/launch ({byts / ms / 1e6:.0f} GB/s of K/V)")
    assert ops.device_status() == 0


def decode_step_case(B: int, launches: int) -> None:
    from llm_serving_engine_b200.llama_decode import LLAMA3_8B, DecodeModel

    m = DecodeModel(LLAMA3_8B, B, 1024, torch.device("cuda"), seed=11, quantize=True, attention="paged")
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        m.step()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        m.step()
    graph.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("step")
    a.record()
    for _ in range(launches):
        graph.replay()
    b.record()
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / launches
    print(f"Llama-3-8B int8 decode step, {B} sequences x 1024 positions: {ms:.3f} ms/step ({B / ms * 1e3:.0f} tokens/s)")
    assert ops.device_status() == 0


def prefill_attention_case(E: int, launches: int) -> None:
    H, H_kv, D, bs, qlen = 32, 8, 128, 16, 2048 // E
    g = torch.Generator(device="cuda").manual_seed(0)
    nbps = -(-qlen // bs)
    nb = E * nbps + 1
    bt = torch.randperm(nb, device="cuda", generator=g)[: E * nbps].view(E, nbps).to(torch.int32)
    i32 = lambda v: torch.tensor(v, dtype=torch.int32, device="cuda")
    cl, off = i32([qlen] * E), i32([0] * E)
    qs, ql = i32([e * qlen for e in range(E)]), i32([qlen] * E)
    kp = torch.randn(nb, bs, H_kv, D, device="cuda", generator=g).to(torch.bfloat16)
    vp = torch.randn(nb, bs, H_kv, D, device="cuda", generator=g).to(torch.bfloat16)
    q = torch.randn(H, E * qlen, D, device="cuda", generator=g).to(torch.bfloat16)
    o = torch.empty_like(q)
    for _ in range(2):
        ops.paged_attention(q, kp, vp, bt, cl, off, qs, ql, bs, qlen, out=o)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(launches):
        ops.paged_attention(q, kp, vp, bt, cl, off, qs, ql, bs, qlen, out=o)
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / launches
    flops = 4.0 * D * H * E * qlen * (qlen + 1) / 2
    print(f"paged attention, {E} x {qlen}-token prefill: {ms * 1e3:.1f} us/launch ({flops / ms / 1e9:.1f} TFLOP/s)")
    assert ops.device_status() == 0


if __name__ == "__main__":
    main()
