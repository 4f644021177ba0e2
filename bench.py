"""Decode benchmark: BASELINE config 4 on 1..8 B200s (one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
    torchrun --nproc-per-node N --master-addr 127.0.0.1 bench.py --gpus N ...

Workload: Qwen3-8B architecture with random-init weights
(seed 0; linear ~N(0, 0.02), norm weights 1, tied embeddings), batch 16, every row
prefilled to 8192 random token ids (seed 0), then greedy decode steps, tensor-parallel by KV
head over N GPUs with an NCCL all-reduce after o_proj and down_proj. One step = one
greedy token for each of the 16 rows = one replay of the captured decode graph.

Prints one JSON line (rank 0): whole-job decode tok/s (device time, max over ranks), the
same through the host-facing step API with pinned host token ids (`e2e`), the roofline of
the dominant kernel (split-KV decode attention: algorithmic K/V bytes per launch over its
measured launch time), the reference's algorithm (the CPU oracle port) timed on this host,
SM clocks sampled during the timed region, and the decode-attention GB/s sweep of BASELINE
config 3 (N=1 only).
"""

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path[:0] = [ROOT, os.path.join(ROOT, "fast-transformer_b200")]

import torch  # noqa: E402

METRIC = "decode-attn HBM GB/s (% of B200 peak); decode tok/s at 1/2/4/8 B200"
PRESET = "qwen3-8b"
BATCH, PROMPT = 16, 8192
FALLBACK_HBM_GBS = 6650.0


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            data = json.load(f)
        return float(data["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


# ------------------------------------------------------------------------------ clocks
class Clocks:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus):
        self.gpus = ",".join(str(g) for g in gpus)
        self.proc = None
        self.path = os.path.join(tempfile.gettempdir(), f"clocks_{os.getpid()}.csv")

    def start(self):
        try:
            self.out = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                                          "-lms", "100", "-i", self.gpus], stdout=self.out, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        time.sleep(0.25)

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.15)
        self.proc.terminate()
        self.proc.wait(timeout=10)
        self.out.close()
        sms, maxes, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 8:
                continue
            try:
                sms.append(float(parts[1]))
                maxes.append(float(parts[2]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[4:8]):
                if flag.lower() == "active":
                    reasons.add(name)
        if not sms:
            return None
        loaded = [s for s in sms if s > 0.5 * max(sms)] or sms
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": max(maxes), "reasons": sorted(reasons),
                "samples": len(sms)}


# ------------------------------------------------------------------------------ CPU side
def cpu_decode_sample(layers_timed=1, repeats=1):
    """The reference's algorithm (the CPU oracle port) for one decode step of config 4 on a
    bounded sample: one Qwen3-8B layer at batch 16 over an 8192-slot cache, plus the LM head
    and argmax; returns (seconds per full 36-layer step, threads, sample text)."""
    from oracle import attention as oatt
    from oracle import pointwise as opw
    import qwen3

    threads = torch.get_num_threads()
    cfg = qwen3.Config.make(**{**qwen3.PRESETS[PRESET], "num_hidden_layers": 1})
    g = torch.Generator().manual_seed(0)
    h, i, d = cfg.hidden_size, cfg.intermediate_size, cfg.head_dim
    hq, hkv = cfg.num_attention_heads, cfg.num_key_value_heads

    def lin(o, n):
        return (torch.randn(o, n, generator=g) * 0.02).to(torch.bfloat16)

    wq, wk, wv, wo = lin(hq * d, h), lin(hkv * d, h), lin(hkv * d, h), lin(h, hq * d)
    wg, wu, wd = lin(i, h), lin(i, h), lin(h, i)
    head = lin(cfg.vocab_size, h)
    ones_h, ones_d = torch.ones(h, dtype=torch.bfloat16), torch.ones(d, dtype=torch.bfloat16)
    keys = torch.randn(BATCH, hkv, PROMPT + 1, d, generator=g).to(torch.bfloat16)
    values = torch.randn(BATCH, hkv, PROMPT + 1, d, generator=g).to(torch.bfloat16)
    hidden = torch.randn(BATCH, 1, h, generator=g).to(torch.bfloat16)
    position = torch.tensor([PROMPT], dtype=torch.int64)
    angle = torch.rand(1, 1, d // 2, generator=g)
    cos = torch.cat((angle, angle), -1).cos().to(torch.bfloat16)
    sin = torch.cat((angle, angle), -1).sin().to(torch.bfloat16)

    def layer():
        normalized, residual = opw.add_rms_norm(hidden, hidden, ones_h, 1e-6)
        packed = torch.cat((opw.linear(normalized, wq), opw.linear(normalized, wk), opw.linear(normalized, wv)), -1)
        query = opw.qk_rope_cache(packed, ones_d, ones_d, 1e-6, 1e-6, cos, sin, position, keys, values, hq)
        att = oatt.decode_attention(query.transpose(1, 2), keys, values, position, 1 / math.sqrt(d))
        out = opw.linear(att.reshape(BATCH, 1, -1), wo)
        normalized, residual = opw.add_rms_norm(out, residual, ones_h, 1e-6)
        gate_up = torch.cat((opw.linear(normalized, wg), opw.linear(normalized, wu)), -1)
        return opw.linear(opw.swiglu(gate_up), wd)

    def tail():
        normalized, _ = opw.add_rms_norm(hidden, hidden, ones_h, 1e-6)
        return opw.argmax(opw.linear(normalized, head))

    layer()  # warm
    t0 = time.perf_counter()
    for _ in range(repeats):
        layer()
    per_layer = (time.perf_counter() - t0) / repeats
    t0 = time.perf_counter()
    tail()
    per_tail = time.perf_counter() - t0
    step = per_layer * qwen3.PRESETS[PRESET]["num_hidden_layers"] + per_tail
    sample = (f"oracle port (torch CPU, fp32 with the reference's bf16 casts): {repeats} x one Qwen3-8B layer "
              f"(B=16, 8192-slot cache, dense split-KV attention) + LM head/argmax once, scaled to 36 layers")
    return step, threads, sample


def reference_arm(args):
    """--impl reference: the reference's decode algorithm on this host's cores (oracle port)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    torch.set_num_threads(os.cpu_count() or 1)
    step_s, threads, sample = cpu_decode_sample(repeats=max(1, min(args.steps, 3)))
    value = BATCH / step_s
    line = {"metric": METRIC, "value": value, "unit": "tok/s", "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_s * 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": config(args),
            "cpu_baseline": {"value": value, "unit": "tok/s", "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def config(args):
    return {"workload": "BASELINE config 4: Qwen3-8B-architecture greedy decode, random init, batch 16, "
                        "8192-token random prompts, TP by KV head",
            "model": "Qwen3-8B architecture (36 layers, hidden 4096, 32/8 heads, D 128, SwiGLU 12288, vocab 151936)",
            "global_batch": BATCH, "seq_len": PROMPT, "parallelism": f"tp{args.gpus}",
            "l2": "per-step inputs (weights + KV, ~35 GB at TP1) exceed the 126 MB L2: no flush needed"}


# ------------------------------------------------------------------------------ GPU side
def attention_roofline(state, layers, repeats=5):
    """Average duration of one decode-attention launch pair (partials + combine) over all
    layer caches, captured in a CUDA graph on the launching stream and timed with events."""
    from kernels.decode_attention import attend
    q = torch.randn(state.batch, state.w.q_heads, 1, state.cfg.head_dim, device=state.device).to(torch.bfloat16)
    out = torch.empty_like(state.attn_out)

    def run():
        for index in range(layers):
            attend(q, state.cache.keys[index], state.cache.values[index], state.position, state.scale,
                   out=out, workspace=state.workspace, ctas=state.ctas)

    run()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.graph(graph, stream=stream):
        run()
    times = []
    with torch.cuda.stream(stream):
        for _ in range(repeats):
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record(stream)
            graph.replay()
            end.record(stream)
            end.synchronize()
            times.append(start.elapsed_time(end) / layers)
    del graph
    return statistics.median(times)


def attention_sweep(peak):
    """ragged decode attention, 32/8 heads, D=128, lengths U[1024, 32768] (seed 0,
    one draw per batch size in order 1, 4, 16, 64); GB/s of K+V+Q+O over graph-timed launches."""
    from kernels.decode_attention import attend, _ctas, workspace_bytes
    gen = torch.Generator().manual_seed(0)
    draws = {b: torch.randint(1024, 32769, (b,), generator=gen).tolist() for b in (1, 4, 16, 64)}
    results = {}
    for batch, lengths in draws.items():
        capacity = max(lengths)
        copies = max(1, min(8, int(math.ceil(400e6 / (2 * batch * 8 * capacity * 128 * 2)))))
        sets = [(torch.randn(batch, 32, 1, 128, device="cuda").to(torch.bfloat16),
                 torch.randn(batch, 8, capacity, 128, device="cuda").to(torch.bfloat16),
                 torch.randn(batch, 8, capacity, 128, device="cuda").to(torch.bfloat16)) for _ in range(copies)]
        position = torch.tensor([n - 1 for n in lengths], dtype=torch.int64, device="cuda")
        ctas = _ctas((torch.device("cuda", torch.cuda.current_device()), batch, 8, capacity, 128))
        ws = torch.zeros(workspace_bytes(batch, 32, 8, 128, ctas), dtype=torch.uint8, device="cuda")
        out = torch.empty(batch, 1, 32, 128, dtype=torch.bfloat16, device="cuda")

        def run():
            for q, k, v in sets:
                attend(q, k, v, position, 1 / math.sqrt(128), out=out, workspace=ws, ctas=ctas)

        run()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            run()
        times = []
        for _ in range(5):
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record()
            graph.replay()
            end.record()
            end.synchronize()
            times.append(start.elapsed_time(end) / copies)
        ms = statistics.median(times)
        nbytes = sum(4096 * n for n in lengths) + batch * 2 * 32 * 128 * 2
        results[f"B{batch}"] = {"us": ms * 1e3, "GB/s": nbytes / ms / 1e6, "frac": nbytes / ms / 1e6 / peak}
        del sets, graph
        torch.cuda.empty_cache()
    return results


def verify_config5(peak):
    """verify attention, B=8, T=5 (causal chain of 5), 32/8 heads, D=128,
    4096-slot prefix + 5 new slots, N(0,1) bf16 (seed 0); graph-timed over L2-cold copies."""
    from kernels.decode_attention import block_attention
    g = torch.Generator(device="cuda").manual_seed(0)
    b, t, hq, hkv, d, cap = 8, 5, 32, 8, 128, 4101
    sets = [(torch.randn(b, t, hq, d, device="cuda", generator=g).to(torch.bfloat16),
             torch.randn(b, hkv, cap, d, device="cuda", generator=g).to(torch.bfloat16),
             torch.randn(b, hkv, cap, d, device="cuda", generator=g).to(torch.bfloat16)) for _ in range(3)]
    position = torch.full((b,), cap - t, dtype=torch.int64, device="cuda")
    chain = torch.full((b,), t, dtype=torch.int64, device="cuda")

    def run():
        for q, k, v in sets:
            block_attention(q, k, v, position, 1 / math.sqrt(d), chain)

    run()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        run()
    times = []
    for _ in range(5):
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        graph.replay()
        end.record()
        end.synchronize()
        times.append(start.elapsed_time(end) / len(sets))
    ms = statistics.median(times)
    nbytes = 2 * b * hkv * cap * d * 2 + 2 * b * t * hq * d * 2
    flops = 4 * b * hq * t * cap * d
    return {"us": ms * 1e3, "GB/s": nbytes / ms / 1e6, "frac": nbytes / ms / 1e6 / peak,
            "useful_TFLOP/s": flops / ms / 1e9, "kernel": "fb_verify_attention (tcgen05)"}


def main():
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=128)
    parser.add_argument("--warmup", type=int, default=3)
    parser.add_argument("--impl", choices=("b200", "reference"), default="b200")
    parser.add_argument("--no-sweep", action="store_true", help="skip the config-3 attention sweep")
    parser.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    args = parser.parse_args()
    if args.warmup < 3:
        parser.error("at least 3 warm-up steps")
    if args.impl == "reference":
        return reference_arm(args)

    import decode as fdecode
    import qwen3
    from kernels import _native

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}: launch N>1 under torchrun")
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    group = None
    if world > 1:
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=device)
        group = torch.distributed.group.WORLD
    peak, peak_kind = peaks()
    cfg = qwen3.Config.make(**qwen3.PRESETS[PRESET])
    weights = qwen3.random_init(cfg, device, seed=0, tp_rank=rank, tp_size=world)
    prompt = torch.randint(0, cfg.vocab_size, (BATCH, PROMPT), generator=torch.Generator().manual_seed(0)).to(device)
    total_steps = args.warmup + args.steps
    # capacity: the prompt, the warm-up and timed steps of both timed loops, plus one spare slot
    state = fdecode.DecodeState(weights, BATCH, PROMPT, 2 * total_steps + 2,
                                comm=fdecode.Communicator(group, world, rank), device=device)
    with torch.inference_mode():
        state.prefill(prompt)
    state.capture()
    _native.device_error()

    def barrier():
        if world > 1:
            torch.distributed.barrier()

    def max_over_ranks(x):
        t = torch.tensor([x], dtype=torch.float64, device=device)
        if world > 1:
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return float(t.item())

    # ---- device-timed decode steps
    for _ in range(args.warmup):
        state.step()
    clocks = Clocks(list(range(world)) if world > 1 else [local]) if rank == 0 else None
    if clocks:
        clocks.start()
    launches_before = _native.launches
    barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("timed")  # `ncu --nvtx --nvtx-include "timed/"` captures these launches
    start.record()
    for _ in range(args.steps):
        state.step()
    end.record()
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    barrier()
    elapsed = max_over_ranks(start.elapsed_time(end))
    clock = clocks.stop() if clocks else None
    ms_per_step = elapsed / args.steps
    value = BATCH / (ms_per_step / 1e3)
    # kernels per step: counted while capturing the step (graph replays launch the same set)
    per_step_launches = state.launches_per_step

    # ---- end to end through the host-facing step: pinned ids in, replay, pinned ids out
    host_in = torch.empty(BATCH, dtype=torch.int64, pin_memory=True)
    host_out = torch.empty(BATCH, dtype=torch.int64, pin_memory=True)
    host_in.copy_(state.token_ids[:, 0].cpu())
    stream = torch.cuda.current_stream()
    for _ in range(args.warmup):
        state.step_host(host_in, host_out)
        stream.synchronize()
        host_in.copy_(host_out)
    barrier()
    torch.cuda.synchronize()
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_start.record()
    for _ in range(args.steps):
        state.step_host(host_in, host_out)
        stream.synchronize()
        host_in.copy_(host_out)
    e_end.record()
    torch.cuda.synchronize()
    barrier()
    e_elapsed = max_over_ranks(e_start.elapsed_time(e_end))
    e2e = {"value": BATCH / (e_elapsed / args.steps / 1e3), "unit": "tok/s",
           "h2d_bytes_per_step": host_in.numel() * host_in.element_size(),
           "d2h_bytes_per_step": host_out.numel() * host_out.element_size()}

    # ---- roofline of the dominant kernel: decode attention over this rank's caches
    attn_ms = attention_roofline(state, cfg.num_hidden_layers)
    valid = int(state.position.item()) + 1  # slots [0, position] the roofline launches attend
    kv_bytes = 2 * BATCH * weights.kv_heads * valid * cfg.head_dim * 2
    qo_bytes = 2 * BATCH * weights.q_heads * cfg.head_dim * 2
    achieved = (kv_bytes + qo_bytes) / (attn_ms / 1e3) / 1e9
    # DRAM traffic of one launch from an ncu capture of this kernel at 16 rows x 8 KV heads x
    # 8320 slots (dram__bytes_read.sum 545.77 MB + dram__bytes_write.sum 4.09 MB), scaled to
    # this launch's valid slots (traffic grows in proportion to the slots streamed)
    traffic = (545.77e6 + 4.09e6) * (valid / 8320) if weights.kv_heads == 8 else None
    roofline = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                "traffic": traffic, "kernel": "fb_decode_attention (per layer)",
                "algorithmic_bytes": kv_bytes + qo_bytes, "launch_us": attn_ms * 1e3,
                "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else "fallback 6.65 TB/s"}
    # per-rank algorithmic bytes of an average timed step: every weight once, K/V of the valid slots
    step_bytes = weights.nbytes_per_step() + state.cache.nbytes_valid(PROMPT + args.warmup + args.steps // 2 + 1)
    step_frac = step_bytes / (ms_per_step / 1e3) / 1e9 / peak
    assert _native.device_error() == 0, "a kernel raised the device error word"
    state.release()
    multicast = bool(state.peers is not None and state.peers.multicast)
    del state
    torch.cuda.empty_cache()

    if world > 1:
        barrier()
        torch.distributed.destroy_process_group()
    if rank != 0:
        return
    line = {"metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (random-init weights and token ids, seed 0)",
            "config": config(args), "e2e": e2e, "roofline": roofline,
            "per_gpu_hbm_frac": step_frac,
            "gpu_launches": per_step_launches * args.steps}
    if clock:
        line["clocks"] = clock
    if world > 1:
        line["allreduce"] = ("flagged fp32 words pushed by the producer (split partials + fb_reduce_push, or the "
                             "projection's epilogue at one split) into every rank's symmetric-memory receive buffer "
                             + ("through the NVSwitch multicast address (multimem.st)" if multicast else
                                "by NVLink peer stores") + "; consumer polls, sums ranks in order + add/RMSNorm")

    if world == 1 and not args.no_sweep:
        line["attention_sweep"] = attention_sweep(peak)
        line["verify_attention_config5"] = verify_config5(peak)
    if world == 1 and not args.no_cpu:
        torch.set_num_threads(os.cpu_count() or 1)
        step_s, threads, sample = cpu_decode_sample()
        line["cpu_baseline"] = {"value": BATCH / step_s, "unit": "tok/s", "cores": threads, "kind": "port",
                                "sample": sample}
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
