"""Run one decode-path kernel (or one eager decode step) at a chosen shape, for Nsight Compute.

    python fast-transformer_b200/profile_kernels.py attention --batch 16 --length 8320
    python fast-transformer_b200/profile_kernels.py linear --m 16 --n 24576 --k 4096 --epilogue 2
    python fast-transformer_b200/profile_kernels.py verify --batch 8 --tokens 5 --length 4101
    python fast-transformer_b200/profile_kernels.py prefill --batch 1 --length 8192
    python fast-transformer_b200/profile_kernels.py forms --tp-size 8 --copies 8
    python fast-transformer_b200/profile_kernels.py step --preset qwen3-8b --batch 16 --length 8192

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
sys.path.insert(0, HERE)

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


def forms(args):
    """Graph-timed per-launch cost of finishing a K-split projection in its own launch (split
    fix-up) against split partials + a consumer kernel, at one tensor-parallel shard's shapes
    (rank 0 of --tp-size, --batch rows): the SwiGLU gate_up, and the o_proj / down_proj
    all-reduce producers pushing into this GPU's own receive buffer (world 1)."""
    import ctypes
    import qwen3
    from kernels import linear as klin
    from kernels._native import check, lib, ptr, stream
    cfg = qwen3.PRESETS[args.preset]
    r, m = args.tp_size, args.batch
    hidden, inter = cfg["hidden_size"], cfg["intermediate_size"] // r
    heads = cfg["num_attention_heads"] // r * cfg["head_dim"]
    epoch = torch.full((1,), 5, dtype=torch.int64, device="cuda")
    recv = torch.zeros(1, 1, m, hidden, dtype=torch.int64, device="cuda")
    peers = (ctypes.c_void_p * 1)(recv.data_ptr())

    def timed(name, n, k, fn):
        x = torch.randn(m, k, device="cuda").bfloat16()
        weights = [(torch.randn(n, k, device="cuda") * 0.02).bfloat16() for _ in range(args.copies)]
        ms = graph_time(lambda: [fn(x, w) for w in weights]) / len(weights)
        print(f"{name} TP-shard 1/{r} M={m} N={n} K={k}: {ms * 1e3:.2f} us per use, {n * k * 2 / ms / 1e6:.0f} GB/s")

    def swiglu(split_consumer):
        return lambda x, w: klin.swiglu_linear(x, w, split_consumer=split_consumer)

    def push(split_consumer, single=False):
        def run(x, w):
            n, k = w.shape
            s = 1 if single else klin.splits_for(m, n, k, x.device, finished=True)
            if s > 1 and split_consumer:
                part = klin.project(x, w, klin.SPLITS_OUT, s)
                check(lib.fb_reduce_push(ptr(part), s, m, n, 1, 0, 0, peers, None, ptr(epoch), stream()), "push")
            else:
                check(lib.fb_linear_allreduce_push(ptr(x), ptr(w), m, n, k, s, 1, 0, 0, peers, None, ptr(epoch),
                                                   stream()), "push")
        return run

    s_gu = klin.splits_for(m, 2 * inter, hidden, torch.device("cuda"), finished=True)
    timed(f"gate_up+SwiGLU fix-up S={s_gu}", 2 * inter, hidden, swiglu(False))
    timed(f"gate_up split partials S={s_gu} + fb_swiglu_blocked", 2 * inter, hidden, swiglu(True))
    for name, k in (("o_proj", heads), ("down_proj", inter)):
        s_p = klin.splits_for(m, hidden, k, torch.device("cuda"), finished=True)
        timed(f"{name} push, one split", hidden, k, push(False, single=True))
        timed(f"{name} push, fix-up S={s_p}", hidden, k, push(False))
        timed(f"{name} split partials S={s_p} + fb_reduce_push", hidden, k, push(True))


def step(args):
    import decode as fdecode
    import qwen3
    cfg = qwen3.Config.make(**qwen3.PRESETS[args.preset])
    # --tp-size N: one rank's shard shapes (rank 0 of N), run alone, for per-kernel times at TP N
    # (the all-reduce consumers then run as the single-rank add+norm)
    if args.finish_in_projection:
        fdecode.FINISH_SPLITS_IN_PROJECTION = True
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
        form = "splits finished in the projections" if fdecode.FINISH_SPLITS_IN_PROJECTION else "split consumers"
        print(f"step {args.preset} TP-shard 1/{args.tp_size} B={args.batch} L={args.length} ({form}): "
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
    parser.add_argument("mode", choices=("attention", "linear", "verify", "prefill", "forms", "step"))
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
    parser.add_argument("--finish-in-projection", action="store_true",
                        help="step: finish K splits inside the projections (split fix-up) instead of in consumer "
                             "kernels (the decode default)")
    parser.add_argument("--copies", type=int, default=2)
    parser.add_argument("--shapes", default="", help="attention: cluster-form shapes to sweep, e.g. 8x2,8x3,16x2")
    parser.add_argument("--launches", type=int, default=2)
    args = parser.parse_args()
    {"attention": attention, "linear": linear, "verify": verify, "prefill": prefill, "forms": forms,
     "step": step}[args.mode](args)


if __name__ == "__main__":
    main()
