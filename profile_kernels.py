"""Run one decode-path kernel (or one eager decode step) at a chosen shape, for Nsight Compute.

    python profile_kernels.py attention --batch 16 --length 8320
    python profile_kernels.py linear --m 16 --n 24576 --k 4096 --epilogue 2
    python profile_kernels.py verify --batch 8 --tokens 5 --length 4101
    python profile_kernels.py prefill --batch 1 --length 8192
    python profile_kernels.py step --preset qwen3-8b --batch 16 --length 8192

Each mode warms up, then runs the measured launches inside the NVTX range "profiled", so
`ncu --nvtx --nvtx-include "profiled/"` captures exactly those; it also prints the CUDA-event
time of the same launches measured without a profiler (graph-replayed, inputs larger than L2).
"""

import argparse
import math
import os
import statistics
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path[:0] = [HERE, os.path.join(HERE, "fast-transformer_b200")]

import torch  # noqa: E402


def graph_time(fn, repeats=5):
    fn()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        fn()
    times = []
    for _ in range(repeats):
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        graph.replay()
        end.record()
        end.synchronize()
        times.append(start.elapsed_time(end))
    return statistics.median(times)


def attention(args):
    from kernels.decode_attention import attend, _ctas, workspace_bytes
    b, hq, hkv, d, n = args.batch, args.q_heads, args.kv_heads, 128, args.length
    sets = [(torch.randn(b, hq, 1, d, device="cuda").bfloat16(), torch.randn(b, hkv, n, d, device="cuda").bfloat16(),
             torch.randn(b, hkv, n, d, device="cuda").bfloat16()) for _ in range(args.copies)]
    position = torch.tensor([n - 1], dtype=torch.int64, device="cuda")
    ctas = _ctas((torch.device("cuda", 0), b, hkv, n, d))
    ws = torch.zeros(workspace_bytes(b, hq, hkv, d, ctas), dtype=torch.uint8, device="cuda")
    out = torch.empty(b, 1, hq, d, dtype=torch.bfloat16, device="cuda")

    def run():
        for q, k, v in sets:
            attend(q, k, v, position, 1 / math.sqrt(d), out=out, workspace=ws, ctas=ctas)

    nbytes = 2 * b * hkv * n * d * 2 + 2 * b * hq * d * 2
    if args.shapes:
        # cluster-form launch shapes (cluster x ring stages), each checked against the automatic choice
        from kernels._native import lib
        run()
        expect = out.clone()
        for shape in args.shapes.split(","):
            cluster, stages = (int(v) for v in shape.split("x"))
            lib.fb_decode_attention_cluster_shape(cluster, stages)
            try:
                ms = graph_time(run) / len(sets)
            except RuntimeError as exc:
                print(f"attention B={b} Hq={hq} Hkv={hkv} L={n} cluster {shape}: not launched ({exc})")
                continue
            finally:
                lib.fb_decode_attention_cluster_shape(0, 0)
            diff = (out.float() - expect.float()).abs().max().item()
            print(f"attention B={b} Hq={hq} Hkv={hkv} L={n} cluster {shape}: {ms * 1e3:.2f} us/launch, "
                  f"{nbytes / ms / 1e6:.0f} GB/s (max |diff| to the automatic shape: {diff:.3g})")
    ms = graph_time(run) / len(sets)
    print(f"attention B={b} Hq={hq} Hkv={hkv} L={n}: {ms * 1e3:.2f} us/launch, {nbytes / ms / 1e6:.0f} GB/s "
          f"({nbytes} algorithmic bytes per launch)")
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_push("profiled")
    for _ in range(args.launches):
        attend(*sets[0], position, 1 / math.sqrt(d), out=out, workspace=ws, ctas=ctas)
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()


def linear(args):
    from kernels.linear import SPLITS_OUT, project, splits_for
    x = torch.randn(args.m, args.k, device="cuda").bfloat16()
    weights = [(torch.randn(args.n, args.k, device="cuda") * 0.02).bfloat16() for _ in range(args.copies)]
    splits = args.splits or splits_for(args.m, args.n, args.k, x.device, finished=args.epilogue != SPLITS_OUT)

    def run():
        for w in weights:
            project(x, w, args.epilogue, splits)

    ms = graph_time(run) / len(weights)
    nbytes = args.n * args.k * 2
    print(f"linear M={args.m} N={args.n} K={args.k} epilogue={args.epilogue} S={splits}: {ms * 1e3:.2f} us, "
          f"{nbytes / ms / 1e6:.0f} GB/s")
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_push("profiled")
    for _ in range(args.launches):
        project(x, weights[0], args.epilogue, splits)
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()


def verify(args):
    """B=8, T=5 (chain 5), 32/8 heads, D=128, 4096-slot prefix + 5 new slots."""
    from kernels.decode_attention import block_attention
    b, t, hq, hkv, d, cap = args.batch, args.tokens, args.q_heads, args.kv_heads, 128, args.length
    sets = [(torch.randn(b, t, hq, d, device="cuda").bfloat16(), torch.randn(b, hkv, cap, d, device="cuda").bfloat16(),
             torch.randn(b, hkv, cap, d, device="cuda").bfloat16()) for _ in range(args.copies)]
    position = torch.full((b,), cap - t, dtype=torch.int64, device="cuda")
    chain = torch.full((b,), t, dtype=torch.int64, device="cuda")

    def run():
        for q, k, v in sets:
            block_attention(q, k, v, position, 1 / math.sqrt(d), chain)

    ms = graph_time(run) / len(sets)
    nbytes = 2 * b * hkv * cap * d * 2 + 2 * b * t * hq * d * 2
    flops = 4 * b * hq * t * cap * d
    print(f"verify B={b} T={t} Hq={hq} Hkv={hkv} L={cap}: {ms * 1e3:.2f} us, {nbytes / ms / 1e6:.0f} GB/s, "
          f"{flops / ms / 1e9:.1f} TFLOP/s useful")
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_push("profiled")
    for _ in range(args.launches):
        block_attention(*sets[0], position, 1 / math.sqrt(d), chain)
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()


def prefill(args):
    """One config-4 prompt row: causal GQA attention over --length tokens, ours vs torch SDPA
    (the reference's own call, library Flash attention) for comparison."""
    from kernels.prefill import prefill_attention
    b, hq, hkv, d, n = args.batch, args.q_heads, args.kv_heads, 128, args.length
    q = torch.randn(b, hq, n, d, device="cuda").bfloat16()
    k = torch.randn(b, hkv, n, d, device="cuda").bfloat16()
    v = torch.randn(b, hkv, n, d, device="cuda").bfloat16()
    scale = 1 / math.sqrt(d)
    flops = 4 * b * hq * d * n * (n + 1) / 2  # causal: QK^T and PV over the lower triangle
    ms = graph_time(lambda: prefill_attention(q, k, v, scale))
    ms_ref = graph_time(lambda: torch.nn.functional.scaled_dot_product_attention(
        q, k, v, is_causal=True, scale=scale, enable_gqa=True))
    print(f"prefill B={b} Hq={hq} Hkv={hkv} T={n}: {ms * 1e3:.1f} us, {flops / ms / 1e9:.1f} TFLOP/s "
          f"(torch SDPA {ms_ref * 1e3:.1f} us, {flops / ms_ref / 1e9:.1f} TFLOP/s)")
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_push("profiled")
    for _ in range(args.launches):
        prefill_attention(q, k, v, scale)
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()


def step(args):
    import decode as fdecode
    import qwen3
    cfg = qwen3.Config.make(**qwen3.PRESETS[args.preset])
    # --tp-size N: one rank's shard shapes (rank 0 of N), run alone, for per-kernel times at TP N
    # (the all-reduce consumers then run as the single-rank add+norm)
    weights = qwen3.random_init(cfg, "cuda", seed=0, tp_rank=0, tp_size=args.tp_size)
    state = fdecode.DecodeState(weights, args.batch, args.length, 8)
    # decode cost does not depend on cache contents: random K/V instead of a prefill
    state.cache.store.normal_()
    state.position.fill_(args.length)
    for _ in range(2):
        state.decode()
        state.position.fill_(args.length)
    torch.cuda.synchronize()
    if args.timed:
        # the captured step, replayed (PDL chains intact), CUDA events around 20 replays
        state.capture()
        for _ in range(3):
            state.position.fill_(args.length)
            state.step()
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(20):
            state.position.fill_(args.length)
            state.step()
        end.record()
        end.synchronize()
        ms = start.elapsed_time(end) / 20
        print(f"step {args.preset} TP-shard 1/{args.tp_size} B={args.batch} L={args.length}: "
              f"{ms * 1e3:.1f} us per captured step ({args.batch / ms * 1e3:.0f} tok/s for this shard alone)")
        state.release()
        return
    torch.cuda.nvtx.range_push("profiled")
    state.decode()
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    print(f"step {args.preset} TP-shard 1/{args.tp_size} B={args.batch} L={args.length}: one eager decode step profiled")


def main():
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("mode", choices=("attention", "linear", "verify", "prefill", "step"))
    parser.add_argument("--batch", type=int, default=16)
    parser.add_argument("--q-heads", type=int, default=32)
    parser.add_argument("--kv-heads", type=int, default=8)
    parser.add_argument("--length", type=int, default=8320)
    parser.add_argument("--tokens", type=int, default=5)
    parser.add_argument("--m", type=int, default=16)
    parser.add_argument("--n", type=int, default=24576)
    parser.add_argument("--k", type=int, default=4096)
    parser.add_argument("--epilogue", type=int, default=3, help="0 bf16, 1 fp32, 2 SwiGLU, 3 split partials")
    parser.add_argument("--splits", type=int, default=0, help="linear: K splits (0: the library's choice)")
    parser.add_argument("--preset", default="qwen3-8b")
    parser.add_argument("--tp-size", type=int, default=1)
    parser.add_argument("--timed", action="store_true", help="step: time the captured step instead of profiling")
    parser.add_argument("--copies", type=int, default=2)
    parser.add_argument("--shapes", default="", help="attention: cluster-form shapes to sweep, e.g. 8x2,8x3,16x2")
    parser.add_argument("--launches", type=int, default=2)
    args = parser.parse_args()
    {"attention": attention, "linear": linear, "verify": verify, "prefill": prefill, "step": step}[args.mode](args)


if __name__ == "__main__":
    main()
