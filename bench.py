"""Decode benchmark: BASELINE config 4 on 1..8 B200s (one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
    torchrun --nproc-per-node N --master-addr 127.0.0.1 bench.py --gpus N ...

Workload: Qwen3-8B architecture with random-init weights
(seed 0; linear ~N(0, 0.02), norm weights 1, tied embeddings), batch 16, every row
prefilled to 8192 random token ids (seed 0), then greedy decode steps, tensor-parallel by KV
head over N GPUs with an all-reduce (flagged-word NVLink peer stores) after o_proj and
down_proj. One step = one greedy token for each of the 16 rows = one replay of the captured
decode graph.

Before any timing a parity gate runs the same step on the 2-layer truncation of the model at
this TP size against the CPU oracle (teacher-forced) and checks graph == eager and that the
ranks agree; a failed gate prints no number.

Prints one JSON line (rank 0): whole-job decode tok/s (device time, max over ranks), the
same through the host-facing step API with pinned host token ids (`e2e`), the roofline of
the dominant kernel (split-KV decode attention: algorithmic K/V bytes per launch over its
measured launch time), SM clocks sampled during the timed region, and at N=1 the other
BASELINE configs (1: decode attention op, 2: Qwen3-0.6B decode, 3: ragged attention sweep,
5: verify attention) and the CPU baseline: the reference's eager path (HF Transformers Qwen3
over a pre-filled DynamicCache) timed on this host's cores.

`--impl reference` prints the CPU baseline alone as the reference arm's line.
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
def host_memory_available():
    """Bytes this process may still allocate on the host: the smaller of the free memory and the
    container's cgroup limit minus its usage."""
    import psutil
    free = psutil.virtual_memory().available
    try:
        limit = open("/sys/fs/cgroup/memory.max").read().strip()
        used = int(open("/sys/fs/cgroup/memory.current").read().strip())
        if limit != "max":
            free = min(free, int(limit) - used)
    except OSError:
        pass
    return free


def _tile(dst, block):
    """Fill ``dst`` with copies of ``block`` (one parallel copy per whole repetition)."""
    flat = dst.view(-1)
    n, size = flat.numel(), block.numel()
    whole = n // size * size
    if whole:
        flat[:whole].view(-1, size).copy_(block[None].expand(whole // size, size))
    if whole < n:
        flat[whole:].copy_(block[:n - whole])


HF_NEED_BYTES = 48 << 30  # 8B bf16 weights (16.4 GB) + a 16 x 8192-slot cache (19.3 GB) + the step's copies


def hf_decode_sample(steps, warmup=1, layers=None):
    """The reference's own eager CPU path for config 4's decode step: HF Transformers'
    Qwen3ForCausalLM (the model the reference engine wraps, engine/engine.py:27-35), bf16, SDPA
    attention, greedy over a DynamicCache pre-filled with 8192 slots per row (BASELINE's CPU plan;
    the pattern of agent/local_cpu/smoke_engine.py:77-86). Whole 36-layer steps at batch 16 on all
    host cores. A 16 x 8192 prefill of an 8B model is impractical on a CPU, so the cache is filled
    with seeded N(0, 1) values instead (decode cost does not depend on them); weights are a seeded
    N(0, 0.02) block tiled over every matrix, norm weights 1, embeddings tied.
    ``layers`` < 36 times a truncated model (the bounded sample of the main line's cpu_baseline)
    and scales its per-layer time to 36 layers, the LM head and argmax timed on their own.
    Returns (seconds per 36-layer step, steps run, threads, sample text), or None when the host
    lacks the memory (about 48 GB for the whole model)."""
    import qwen3
    total_layers = qwen3.PRESETS[PRESET]["num_hidden_layers"]
    layers = layers or total_layers
    if host_memory_available() < HF_NEED_BYTES * layers / total_layers + (4 << 30):
        return None
    import warnings
    from transformers import DynamicCache, Qwen3Config, Qwen3ForCausalLM
    from transformers.initialization import no_init_weights
    warnings.filterwarnings("ignore")
    torch.set_num_threads(os.cpu_count() or 1)
    preset = {**qwen3.PRESETS[PRESET], "num_hidden_layers": layers}
    cfg = Qwen3Config(**preset, max_position_embeddings=40960)
    cfg._attn_implementation = "sdpa"
    default = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    try:
        with no_init_weights():
            model = Qwen3ForCausalLM(cfg)
    finally:
        torch.set_default_dtype(default)
    model.eval()
    g = torch.Generator().manual_seed(0)
    block = (torch.randn(1 << 24, generator=g) * 0.02).to(torch.bfloat16)
    with torch.no_grad():
        model.lm_head.weight = model.model.embed_tokens.weight  # tied embeddings
        for name, param in model.named_parameters():
            if name.endswith("norm.weight"):
                param.fill_(1.0)
            else:
                _tile(param.data, block)
        cache = DynamicCache(config=cfg)
        kv = torch.randn(1 << 24, generator=g).to(torch.bfloat16)
        hkv, d = preset["num_key_value_heads"], preset["head_dim"]
        for layer in range(preset["num_hidden_layers"]):
            k = torch.empty(BATCH, hkv, PROMPT, d, dtype=torch.bfloat16)
            v = torch.empty_like(k)
            _tile(k, kv)
            _tile(v, kv)
            cache.update(k, v, layer)
        ids = torch.randint(0, preset["vocab_size"], (BATCH, 1), generator=g)
    times, head_times = [], []
    with torch.inference_mode():
        for step in range(warmup + steps):
            t0 = time.perf_counter()
            logits = model(input_ids=ids, past_key_values=cache, use_cache=True).logits
            ids = logits[:, -1].argmax(-1, keepdim=True)
            if step >= warmup:
                times.append(time.perf_counter() - t0)
            if layers < total_layers:
                hidden = torch.randn(BATCH, 1, preset["hidden_size"], generator=g).to(torch.bfloat16)
                t0 = time.perf_counter()
                model.lm_head(model.model.norm(hidden))[:, -1].argmax(-1)
                if step >= warmup:
                    head_times.append(time.perf_counter() - t0)
    del model, cache
    step_s = statistics.median(times)
    if layers < total_layers:
        head = statistics.median(head_times)
        step_s = (step_s - head) * total_layers / layers + head
        sample = (f"HF Transformers Qwen3ForCausalLM eager (bf16, SDPA), the reference engine's model, truncated to "
                  f"{layers} of {total_layers} layers: {steps} greedy steps at batch 16 over a DynamicCache "
                  f"pre-filled to 8192 slots (seeded N(0,1) K/V), median step, the layers' time scaled to "
                  f"{total_layers} layers plus the final norm, LM head and argmax timed alone")
    else:
        sample = (f"HF Transformers Qwen3ForCausalLM eager (bf16, SDPA), the reference engine's model: {steps} whole "
                  f"{total_layers}-layer greedy steps at batch 16 over a DynamicCache pre-filled to 8192 slots "
                  f"(seeded N(0,1) K/V instead of a prefill), after {warmup} warm-up step; median step")
    return step_s, steps, torch.get_num_threads(), sample


def port_decode_sample(repeats=1):
    """Fallback when the host cannot hold the HF model and cache: the oracle port (torch CPU, fp32
    with the reference's bf16 casts) for one Qwen3-8B layer at batch 16 over an 8192-slot cache
    plus the LM head and argmax, scaled to 36 layers. Returns (seconds per step, threads, sample)."""
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
    sample = (f"oracle port (torch CPU, fp32 with the reference's bf16 casts; the host lacked the ~48 GB the HF "
              f"model and cache need): {repeats} x one Qwen3-8B layer (B=16, 8192-slot cache) + LM head/argmax "
              f"once, scaled to 36 layers")
    return step, threads, sample


def cpu_baseline(steps, layers=None):
    """(tok/s, steps run, threads, kind, sample, seconds per step) of the CPU reference path on
    this host: HF eager Qwen3 (whole steps, or ``layers`` of them scaled), else the oracle port."""
    got = hf_decode_sample(steps, layers=layers)
    if got is not None:
        step_s, ran, threads, sample = got
        return BATCH / step_s, ran, threads, "reference", sample, step_s
    torch.set_num_threads(os.cpu_count() or 1)
    step_s, threads, sample = port_decode_sample()
    return BATCH / step_s, 1, threads, "port", sample, step_s


def reference_arm(args):
    """--impl reference: the reference's eager CPU decode on this host's cores (rank 0 only)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    steps = max(3, min(args.steps, 5))
    value, ran, threads, kind, sample, step_s = cpu_baseline(steps)
    line = {"metric": METRIC, "value": value, "unit": "tok/s", "impl": "reference", "n_gpus": args.gpus,
            "steps": ran, "warmup": 1, "ms_per_step": step_s * 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": config(args),
            "cpu_baseline": {"value": value, "unit": "tok/s", "cores": threads, "kind": kind, "sample": sample},
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


def graph_time_ms(run, repeats=5):
    """Median device time of one replay of ``run`` captured in a CUDA graph (CUDA events on the
    replaying stream, after one eager warm-up pass)."""
    run()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        run()
    times = []
    for _ in range(repeats):
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        graph.replay()
        end.record()
        end.synchronize()
        times.append(start.elapsed_time(end))
    del graph
    return statistics.median(times)


def config1_attention(peak):
    """decode attention, batch 1, 16/8 heads (G=2), D=128, 2048 valid slots,
    N(0,1) bf16 (seed 0), scale 1/sqrt(128); BASELINE's 8 KV splits (the cluster form with 8 CTAs
    per (row, KV head) pair, each streaming 1/8 of the slots) and the kernel's own split choice.
    The north-star target (>= 80% of HBM peak) applies at >= 8k slots, so the same head shape is
    also timed at 8192, 16384 and 32768 slots (the kernel's own choice). Graph-timed over enough
    cache copies that every launch reads from HBM (> L2)."""
    from kernels._native import lib
    from kernels.decode_attention import _ctas, attend, workspace_bytes
    results = {}
    for length in (2048, 8192, 16384, 32768):
        kv_bytes = 2 * 8 * length * 128 * 2
        copies = max(2, int(math.ceil(400e6 / kv_bytes)))
        g = torch.Generator(device="cuda").manual_seed(0)
        q = torch.randn(1, 16, 1, 128, device="cuda", generator=g).to(torch.bfloat16)
        sets = [(torch.randn(1, 8, length, 128, device="cuda", generator=g).to(torch.bfloat16),
                 torch.randn(1, 8, length, 128, device="cuda", generator=g).to(torch.bfloat16)) for _ in range(copies)]
        position = torch.tensor([length - 1], dtype=torch.int64, device="cuda")
        ctas = _ctas((torch.device("cuda", torch.cuda.current_device()), 1, 8, length, 128))
        ws = torch.zeros(workspace_bytes(1, 16, 8, 128, ctas), dtype=torch.uint8, device="cuda")
        out = torch.empty(1, 1, 16, 128, dtype=torch.bfloat16, device="cuda")

        def run():
            for k, v in sets:
                attend(q, k, v, position, 1 / math.sqrt(128), out=out, workspace=ws, ctas=ctas)

        nbytes = kv_bytes + 2 * 16 * 128 * 2
        forms = [("auto", None)] + ([("8 splits", (8, 4))] if length == 2048 else [])
        for name, shape in forms:
            if shape is not None:
                assert lib.fb_decode_attention_cluster_shape(*shape) == 0
            try:
                ms = graph_time_ms(run) / copies
            finally:
                lib.fb_decode_attention_cluster_shape(0, 0)
            results[f"L{length} {name}"] = {"us": ms * 1e3, "GB/s": nbytes / ms / 1e6, "frac": nbytes / ms / 1e6 / peak}
        del sets
        torch.cuda.empty_cache()
    return {"workload": "BASELINE config 1: B=1, 16/8 heads, D=128, 2048 slots, N(0,1) bf16 seed 0 (plus the "
                        "same head shape at 8k-32k slots)", "algorithmic_bytes_L2048": 2 * 8 * 2048 * 128 * 2 + 8192,
            "results": results}


def config2_decode(peak, new_tokens=256, prompt_length=512):
    """Qwen3-0.6B architecture (random init, seed 0), batch 1, a 512-token
    random prompt, 256 greedy tokens on one GPU: the first from the prefill, then 255 replays of
    the captured decode step, device-timed. Per-step roofline: every weight once plus the K/V of
    the valid slots (mean over the steps) per step time."""
    import decode as fdecode
    import qwen3
    cfg = qwen3.Config.make(**qwen3.PRESETS["qwen3-0.6b"])
    weights = qwen3.random_init(cfg, "cuda", seed=0)
    prompt = torch.randint(0, cfg.vocab_size, (1, prompt_length), generator=torch.Generator().manual_seed(0))
    state = fdecode.DecodeState(weights, 1, prompt_length, new_tokens + 8)
    with torch.inference_mode():
        state.prefill(prompt.cuda())
    state.capture()
    steps = new_tokens - 1
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        state.step()
    end.record()
    end.synchronize()
    ms = start.elapsed_time(end) / steps
    state.release()
    step_bytes = weights.nbytes_per_step() + state.cache.nbytes_valid(prompt_length + 1 + steps // 2)
    del state, weights
    torch.cuda.empty_cache()
    return {"workload": "BASELINE config 2: Qwen3-0.6B architecture, random init seed 0, batch 1, 512-token "
                        "prompt, 256 greedy tokens, 1 GPU", "value": 1e3 / ms, "unit": "tok/s", "ms_per_step": ms,
            "roofline": {"bound": "hbm", "algorithmic_bytes_per_step": step_bytes,
                         "achieved": step_bytes / ms / 1e6, "peak": peak, "unit": "GB/s",
                         "frac": step_bytes / ms / 1e6 / peak}}


def parity_gate(comm, rank, world, device):
    """Correctness before any number: the decode step at this tensor-parallel size on the real
    Qwen3-8B architecture truncated to 2 layers (random init, seed 1, this rank's shard), batch
    16, 16-token random prompts, 4 greedy tokens.
      - the captured graph's tokens equal the eager step's;
      - every rank holds the same token ids;
      - rank 0 runs the CPU oracle (oracle/model.py, the reference's arithmetic) on the unsharded
        weights, teacher-forced on the GPU's tokens: logits within 2e-2 of the logit scale and the
        chosen token's gap to the row maximum within max(0.02, 2e-2 of the scale).
    Returns (ok, details); every rank gets rank 0's verdict."""
    import decode as fdecode
    import qwen3
    from oracle import model as omodel
    cfg = qwen3.Config.make(**{**qwen3.PRESETS[PRESET], "num_hidden_layers": 2})
    weights = qwen3.random_init(cfg, device, seed=1, tp_rank=rank, tp_size=world)
    prompt = torch.randint(0, cfg.vocab_size, (BATCH, 16), generator=torch.Generator().manual_seed(1))
    steps = 4
    eager = fdecode.DecodeState(weights, BATCH, 16, steps + 4, comm=comm, device=device)
    tokens, logits = fdecode.greedy(eager, prompt.to(device), steps)
    graph = fdecode.DecodeState(weights, BATCH, 16, steps + 4, comm=comm, device=device)
    graph.prefill(prompt.to(device))
    replayed = [graph.token_ids[:, 0].clone()]
    graph.capture()
    for _ in range(steps - 1):
        graph.step()
        replayed.append(graph.token_ids[:, 0].clone())
    torch.cuda.synchronize()
    graph.release()
    checks = {"graph == eager": bool(torch.equal(torch.stack(replayed, 1), tokens))}
    if world > 1:
        gathered = [torch.empty_like(tokens) for _ in range(world)]
        torch.distributed.all_gather(gathered, tokens)
        checks["ranks agree"] = all(bool(torch.equal(t, gathered[0])) for t in gathered)
    detail = {}
    if rank == 0:
        full = qwen3.random_init(cfg, device, seed=1)
        model = omodel.Model(omodel.Config(**qwen3.PRESETS[PRESET] | {"num_hidden_layers": 2}),
                             qwen3.to_state_dict(full))
        del full
        cache = model.new_cache(BATCH, 16 + steps)
        expect = [model.prefill(prompt, cache)]
        host_tokens = tokens.cpu()
        for step in range(steps - 1):
            expect.append(model.decode(host_tokens[:, step], 16 + step, cache))
        expect = torch.stack(expect, 1).float()
        got = logits.cpu()
        scale = float(expect.abs().max())
        err = float((got - expect).abs().max())
        chosen = expect.gather(-1, host_tokens[..., None])[..., 0]
        gap = float((expect.max(-1).values - chosen).max())
        checks["logits vs oracle"] = err <= 2e-2 * scale
        checks["teacher-forced gap"] = gap <= max(0.02, 2e-2 * scale)
        detail = {"max_abs_err": err, "logit_scale": scale, "max_gap": gap}
    del eager, graph, weights
    torch.cuda.empty_cache()
    verdict = torch.tensor([1 if all(checks.values()) else 0], device=device)
    if world > 1:
        torch.distributed.broadcast(verdict, 0)
    return bool(verdict.item()), {"checks": checks, **detail}


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
    comm = fdecode.Communicator(group, world, rank)
    parity_ok, parity = parity_gate(comm, rank, world, device)
    if not parity_ok:
        if world > 1:
            torch.distributed.destroy_process_group()
        raise SystemExit(f"parity gate failed, no number printed: {json.dumps(parity)}")
    cfg = qwen3.Config.make(**qwen3.PRESETS[PRESET])
    weights = qwen3.random_init(cfg, device, seed=0, tp_rank=rank, tp_size=world)
    prompt = torch.randint(0, cfg.vocab_size, (BATCH, PROMPT), generator=torch.Generator().manual_seed(0)).to(device)
    total_steps = args.warmup + args.steps
    # capacity: the prompt, the warm-up and timed steps of both timed loops, plus one spare slot
    state = fdecode.DecodeState(weights, BATCH, PROMPT, 2 * total_steps + 2, comm=comm, device=device)
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
    # 8320 slots (dram__bytes_read.sum 545.79 MB + dram__bytes_write.sum 5.54 MB), scaled to
    # this launch's valid slots (traffic grows in proportion to the slots streamed)
    traffic = (545.79e6 + 5.54e6) * (valid / 8320) if weights.kv_heads == 8 else None
    roofline = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                "traffic": traffic, "kernel": "fb_decode_attention (per layer)",
                "algorithmic_bytes": kv_bytes + qo_bytes, "launch_us": attn_ms * 1e3,
                "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else "fallback 6.65 TB/s"}
    # per-rank algorithmic bytes of an average timed step: every weight once, K/V of the valid slots
    step_bytes = weights.nbytes_per_step() + state.cache.nbytes_valid(PROMPT + args.warmup + args.steps // 2 + 1)
    step_frac = step_bytes / (ms_per_step / 1e3) / 1e9 / peak
    assert _native.device_error() == 0, "a kernel raised the device error word"
    state.release()
    del state
    torch.cuda.empty_cache()

    # ---- N > 1: the same shard alone (no all-reduce; its consumers run as the single-rank
    # add+RMSNorm), captured and replayed like the timed step. The rest of the step is the
    # all-reduce traffic, its polling and the ranks' skew.
    step_split = None
    if world > 1:
        alone = fdecode.DecodeState(weights, BATCH, PROMPT, 2 * total_steps + 2, device=device)
        alone.cache.store.normal_()  # decode cost does not depend on the cache contents
        alone.position.fill_(PROMPT)
        with torch.inference_mode():
            alone.decode()
        alone.capture()
        for _ in range(args.warmup):
            alone.step()
        barrier()
        torch.cuda.synchronize()
        a_start, a_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a_start.record()
        for _ in range(args.steps):
            alone.step()
        a_end.record()
        torch.cuda.synchronize()
        barrier()
        alone_ms = max_over_ranks(a_start.elapsed_time(a_end)) / args.steps
        assert _native.device_error() == 0, "a kernel raised the device error word"
        alone.release()
        del alone
        torch.cuda.empty_cache()
        step_split = {"step_us": ms_per_step * 1e3, "shard_alone_us": alone_ms * 1e3,
                      "allreduce_and_skew_us": (ms_per_step - alone_ms) * 1e3,
                      "how": "shard alone = this rank's 1/N of every projection and KV head, no all-reduce, "
                             "graph-replayed like the timed step; max over ranks"}

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
            "gpu_launches": per_step_launches * args.steps,
            "parity": "ok", "parity_gate": parity}
    if clock:
        line["clocks"] = clock
    if world > 1:
        if fdecode.ALLREDUCE_FORM == "push":
            line["allreduce"] = ("push form over NVLink peer stores: fb_allreduce_push sums the projection's split-K "
                                 "partials and stores each fp32 value as a flagged word into every rank's receive "
                                 "slab; fb_allreduce_sum_add_rmsnorm polls all slabs, sums the ranks in rank order "
                                 "and applies add+RMSNorm (one NVLink phase)")
        else:
            line["allreduce"] = ("owner-computes over NVLink peer stores: fb_reduce_scatter_push stores each summed "
                                 "fp32 value only to the rank owning its column slice; fb_allreduce_add_rmsnorm sums "
                                 "the ranks per slice, adds the residual, all-gathers the summed rows and per-slice "
                                 "sums of squares and applies the RMSNorm on every rank (two NVLink phases)")
        line["step_split"] = step_split

    if world == 1 and not args.no_sweep:
        line["attention_sweep"] = attention_sweep(peak)
        line["verify_attention_config5"] = verify_config5(peak)
        line["config1_attention"] = config1_attention(peak)
        line["config2_qwen3_0_6b"] = config2_decode(peak)
    if world == 1 and not args.no_cpu:
        value_cpu, ran, threads, kind, sample, _ = cpu_baseline(2, layers=4)
        line["cpu_baseline"] = {"value": value_cpu, "unit": "tok/s", "cores": threads, "kind": kind,
                                "sample": sample, "steps": ran}
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
