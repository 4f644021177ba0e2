"""GPU parity of each CUDA kernel against the reference's own outputs (golden fixtures made by
running the reference's code) and the CPU oracle, at the reference's tolerances
(agent/verify_gpu.py) and BASELINE's (2e-2 abs/rel for bf16 attention outputs)."""

import math
import os
from types import SimpleNamespace

import pytest
import torch

import cases
from oracle import attention as oatt
from oracle import pointwise as opw

pytestmark = pytest.mark.gpu
GOLDEN = os.path.dirname(os.path.abspath(cases.__file__))
DEV = "cuda"


def load(family):
    return torch.load(os.path.join(GOLDEN, f"{family}.pt"), weights_only=False)


@pytest.fixture(autouse=True)
def _no_device_errors():
    from kernels import _native
    _native.device_error()
    yield
    assert _native.device_error() == 0, "a kernel raised its device error word"


def ulps(a, b):
    return (a.contiguous().view(torch.int16).int() - b.contiguous().view(torch.int16).int()).abs()


# ------------------------------------------------------------------ decode attention
@pytest.mark.parametrize("case", cases.DECODE_CASES, ids=[c[0] for c in cases.DECODE_CASES])
def test_decode_attention_matches_reference(case):
    from kernels.decode_attention import decode_attention
    fx = load("decode")[case[0]]
    q, k, v, position, scale = cases.decode_inputs(case)
    assert cases.digest(q, k, v, position) == fx["digest"]
    out = decode_attention(q.to(DEV), k.to(DEV), v.to(DEV), position.to(DEV), scale).cpu()
    assert out.shape == (q.shape[0], 1, q.shape[1], q.shape[3])
    assert torch.isfinite(out.float()).all()
    # reference kernel output; the reference's own decode tolerance (verify_gpu.py:172)
    torch.testing.assert_close(out.float(), fx["out"].float(), atol=0.03125, rtol=0.01)
    # BASELINE tolerance against the oracle
    oracle = oatt.decode_attention(q, k, v, position, scale, splits=8 if case[0] == "c1" else None)
    torch.testing.assert_close(out.float(), oracle.float(), atol=2e-2, rtol=2e-2)


def _ragged(batch, q_heads, kv_heads, dim, lengths, seed, poison=True):
    g = torch.Generator(device=DEV).manual_seed(seed)
    capacity = int(max(lengths))
    q = torch.randn(batch, q_heads, 1, dim, device=DEV, generator=g).bfloat16()
    k = torch.randn(batch, kv_heads, capacity, dim, device=DEV, generator=g).bfloat16()
    v = torch.randn(batch, kv_heads, capacity, dim, device=DEV, generator=g).bfloat16()
    if poison:
        for b, n in enumerate(lengths):
            k[b, :, n:] = float("nan")
            v[b, :, n:] = float("nan")
    position = torch.tensor([n - 1 for n in lengths], dtype=torch.int64, device=DEV)
    return q, k, v, position


def torch_fp32_decode(q, k, v, lengths, scale):
    """Plain PyTorch fp32 reference (GPU) for large shapes: masked softmax per row."""
    batch, q_heads, _, dim = q.shape
    kv_heads = k.shape[1]
    groups = q_heads // kv_heads
    out = torch.empty(batch, 1, q_heads, dim, device=q.device)
    for b, n in enumerate(lengths):
        qq = q[b, :, 0].float().view(kv_heads, groups, dim)
        kk = k[b, :, :n].float()
        vv = v[b, :, :n].float()
        s = torch.einsum("hgd,hnd->hgn", qq, kk) * scale
        p = torch.softmax(s, -1)
        out[b, 0] = torch.einsum("hgn,hnd->hgd", p, vv).reshape(q_heads, dim)
    return out


@pytest.mark.parametrize("batch", [1, 4, 16, 64])
def test_decode_attention_config3_ragged(batch):
    """32/8 heads, D=128, lengths U[1024, 32768] from seed 0, NaN past each length."""
    from kernels.decode_attention import decode_attention
    gen = torch.Generator().manual_seed(0)
    draws = {}
    for b in (1, 4, 16, 64):  # one draw per B, in that order
        draws[b] = torch.randint(1024, 32769, (b,), generator=gen).tolist()
    lengths = draws[batch]  # all rows, B = 64 included (~9 GB of K/V at the longest draw)
    q, k, v, position = _ragged(batch, 32, 8, 128, lengths, seed=batch)
    out = decode_attention(q, k, v, position, 1 / math.sqrt(128))
    expect = torch_fp32_decode(q, k, v, lengths, 1 / math.sqrt(128))
    assert torch.isfinite(out.float()).all()
    torch.testing.assert_close(out.float(), expect, atol=2e-2, rtol=2e-2)


def test_decode_attention_long_and_tiny_lengths():
    """Scalar position at L >= 8k (the >= 80% roofline regime), plus lengths 1 and 63/64/65."""
    from kernels.decode_attention import decode_attention
    for lengths in ([8192], [32768], [1], [63, 64, 65, 1]):
        batch = len(lengths)
        q, k, v, position = _ragged(batch, 16, 8, 128, lengths, seed=len(lengths) + lengths[0])
        if len(set(lengths)) == 1:
            position = position[:1].contiguous()
        out = decode_attention(q, k, v, position, 1 / math.sqrt(128))
        torch.testing.assert_close(out.float(), torch_fp32_decode(q, k, v, lengths, 1 / math.sqrt(128)),
                                   atol=2e-2, rtol=2e-2)


@pytest.mark.parametrize("batch,q_heads,kv_heads,dim,length", [
    (16, 4, 1, 128, 8193),    # a TP8 shard of config 4: clusters of 8
    (16, 8, 2, 128, 4000),    # TP4: clusters of 4
    (2, 8, 2, 64, 100),       # 2 tiles over 8 ranks: empty slices
    (3, 32, 8, 128, 1),       # one valid slot
    (1, 8, 1, 128, 30000),
])
def test_decode_attention_cluster_form(batch, q_heads, kv_heads, dim, length):
    """A shared position over few (row, KV head) pairs takes the cluster form (per-pair DSMEM
    merge): it must match the fp32 reference like the persistent form, which the same lengths
    given per row still take, and ignore NaN past the valid length."""
    from kernels.decode_attention import decode_attention
    lengths = [length] * batch
    q, k, v, position = _ragged(batch, q_heads, kv_heads, dim, lengths, seed=batch * 7 + length)
    shared = position[:1].contiguous()
    cluster = decode_attention(q, k, v, shared, 1 / math.sqrt(dim))
    persistent = decode_attention(q, k, v, position, 1 / math.sqrt(dim))
    expect = torch_fp32_decode(q, k, v, lengths, 1 / math.sqrt(dim))
    assert torch.isfinite(cluster.float()).all()
    torch.testing.assert_close(cluster.float(), expect, atol=2e-2, rtol=2e-2)
    torch.testing.assert_close(cluster.float(), persistent.float(), atol=2e-2, rtol=2e-2)
    again = decode_attention(q, k, v, shared, 1 / math.sqrt(dim))
    assert torch.equal(cluster, again)  # deterministic


@pytest.mark.parametrize("shape", [(2, 2), (4, 4), (8, 2), (8, 3), (16, 2), (16, 3), (9, 4), (6, 3), (13, 2)])
def test_decode_attention_cluster_shapes(shape):
    """Every cluster-form launch shape (cluster size x ring depth, fb_decode_attention_cluster_shape)
    against the fp32 reference at a TP8 shard (16 rows x 1 KV head x 4 query heads, 8193 slots,
    NaN past the length) and a ragged tile count (1000 slots); a shape that does not fit one
    wave returns FB_ERR_SHAPE."""
    from kernels._native import lib
    from kernels.decode_attention import decode_attention
    cluster, stages = shape
    for batch, q_heads, kv_heads, length in ((16, 4, 1, 8193), (3, 16, 2, 1000)):
        lengths = [length] * batch
        q, k, v, position = _ragged(batch, q_heads, kv_heads, 128, lengths, seed=cluster * 10 + stages + length)
        shared = position[:1].contiguous()
        expect = torch_fp32_decode(q, k, v, lengths, 1 / math.sqrt(128))
        assert lib.fb_decode_attention_cluster_shape(cluster, stages) == 0
        try:
            out = decode_attention(q, k, v, shared, 1 / math.sqrt(128))
        except RuntimeError as exc:
            assert "-2" in str(exc) or "SHAPE" in str(exc).upper(), exc
            continue
        finally:
            lib.fb_decode_attention_cluster_shape(0, 0)
        assert torch.isfinite(out.float()).all()
        torch.testing.assert_close(out.float(), expect, atol=2e-2, rtol=2e-2)


def test_decode_attention_groups_above_eight_are_refused():
    """GQA groups above 8 query heads per KV head are outside the kernel's contract (G <= 8,
    the mma N): the C entry point returns FB_ERR_SHAPE and writes nothing."""
    from kernels._native import lib, ptr, stream
    from kernels.decode_attention import _ctas, workspace_bytes
    q, k, v, position = _ragged(4, 16, 1, 128, [65] * 4, seed=93)
    out = torch.full((4, 1, 16, 128), 3.0, dtype=torch.bfloat16, device=DEV)
    ctas = _ctas((q.device, 4, 1, k.shape[2], 128))
    ws = torch.zeros(workspace_bytes(4, 16, 1, 128, ctas), dtype=torch.uint8, device=DEV)
    status = lib.fb_decode_attention(ptr(q), ptr(k), ptr(v), ptr(position[:1].contiguous()), 0, ptr(out), ptr(ws),
                                     ws.numel(), 4, 16, 1, 128, k.shape[2], 0.088, ctas, stream())
    torch.cuda.synchronize()
    assert status == -2
    assert bool((out == 3.0).all())


def test_decode_attention_forced_shape_beyond_one_wave_is_refused():
    """A forced cluster shape whose clusters cannot all be resident at once (16 pairs x clusters
    of 16 CTAs with the one-CTA-per-SM ring: 256 CTAs) returns FB_ERR_SHAPE and launches nothing:
    the output keeps its sentinel."""
    from kernels._native import lib, ptr, stream
    from kernels.decode_attention import _ctas, workspace_bytes
    q, k, v, position = _ragged(16, 4, 1, 128, [2048] * 16, seed=77)
    shared = position[:1].contiguous()
    out = torch.full((16, 1, 4, 128), 3.0, dtype=torch.bfloat16, device=DEV)
    ctas = _ctas((q.device, 16, 1, k.shape[2], 128))
    ws = torch.zeros(workspace_bytes(16, 4, 1, 128, ctas), dtype=torch.uint8, device=DEV)
    assert lib.fb_decode_attention_cluster_shape(16, 4) == 0
    try:
        status = lib.fb_decode_attention(ptr(q), ptr(k), ptr(v), ptr(shared), 0, ptr(out), ptr(ws), ws.numel(), 16, 4,
                                         1, 128, k.shape[2], 0.088, ctas, stream())
    finally:
        lib.fb_decode_attention_cluster_shape(0, 0)
    torch.cuda.synchronize()
    assert status == -2
    assert bool((out == 3.0).all())


def test_decode_attention_graph_capture_and_determinism():
    from kernels.decode_attention import decode_attention
    q, k, v, position = _ragged(2, 32, 8, 128, [5000, 777], seed=5, poison=False)
    position[0] -= 1  # leave room to advance
    eager = decode_attention(q, k, v, position, 0.088)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        captured = decode_attention(q, k, v, position, 0.088)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(eager, captured)  # same partition, same order: bitwise deterministic
    position.add_(1)  # the device-side position moves; the replay follows it
    graph.replay()
    again = decode_attention(q, k, v, position, 0.088)
    torch.cuda.synchronize()
    assert torch.equal(again, captured)


# ------------------------------------------------------------------ QK norm + RoPE + append
@pytest.mark.parametrize("case", cases.ROPE_CASES, ids=[c[0] for c in cases.ROPE_CASES])
def test_qk_rope_cache_matches_reference(case):
    from kernels.merged import Split
    from kernels.qk_rope import qk_rope_cache
    fx = load("rope")[case[0]]
    x = cases.rope_inputs(case)
    packed = x["packed"].to(DEV)
    batch = x["keys"].shape[0]
    if packed.dtype == torch.float32:
        packed = Split(packed, (batch, packed.shape[1] // batch, packed.shape[2]))
    q_norm = SimpleNamespace(weight=x["q_weight"].to(DEV), variance_epsilon=x["q_eps"])
    k_norm = SimpleNamespace(weight=x["k_weight"].to(DEV), variance_epsilon=x["k_eps"])
    keys, values = x["keys"].to(DEV), x["values"].to(DEV)
    phases = x["phases"].to(DEV) if x["phases"] is not None else None
    query = qk_rope_cache(packed, q_norm, k_norm, x["cos"].to(DEV), x["sin"].to(DEV), x["position"].to(DEV),
                          keys, values, x["q_heads"], prefill=x["prefill"], rows=x["rows"], phases=phases)
    query = query.transpose(1, 2).contiguous().cpu()
    keys, values = keys.cpu(), values.cpu()
    # V is a copy: bit-exact, and every slot the step must not write keeps its sentinel
    assert torch.equal(values, fx["values"])
    written = fx["keys"] != 17
    assert torch.equal(keys[~written], fx["keys"][~written])
    # K (the cache contents) and Q: bit-exact (the sum of squares is added in the reference's
    # eager order, every step correctly rounded)
    for name, actual, expected in (("query", query, fx["query"]), ("keys", keys, fx["keys"])):
        differ = (actual != expected).nonzero()
        assert differ.numel() == 0, f"{name}: {differ.shape[0]} elements differ, first {differ[:4].tolist()}"


# ------------------------------------------------------------------ norms, SwiGLU, projections, argmax
def test_rms_norm_family_matches_reference():
    from kernels.rmsnorm import add_rms_norm, embed_rms_norm, rms_norm
    fx = load("pointwise")
    for case in cases.NORM_CASES:
        x, residual, weight, eps, table, ids = cases.norm_inputs(case)
        f = fx[case[0]]
        got = rms_norm(x.to(DEV), weight.to(DEV), eps).cpu()
        assert (got == f["rms"]).float().mean() >= 0.999 and ulps(got, f["rms"]).max() <= 2
        added, summed = add_rms_norm(x.to(DEV), residual.to(DEV), weight.to(DEV), eps)
        assert torch.equal(summed.cpu(), f["sum"])  # the bf16 residual sum is exact
        assert (added.cpu() == f["add"]).float().mean() >= 0.999 and ulps(added.cpu(), f["add"]).max() <= 2
        embedded, hidden = embed_rms_norm(ids.to(DEV), table.to(DEV), weight.to(DEV), eps)
        assert torch.equal(hidden.cpu(), f["hidden"])
        assert (embedded.cpu() == f["embed"]).float().mean() >= 0.999


def test_add_rms_norm_split_input():
    from kernels.merged import Split
    from kernels.rmsnorm import add_rms_norm
    g = torch.Generator().manual_seed(7)
    partial = torch.randn(3, 4, 1024, generator=g)
    residual = torch.randn(4, 1, 1024, generator=g).bfloat16()
    weight = torch.randn(1024, generator=g).bfloat16()
    out, summed = add_rms_norm(Split(partial.to(DEV), (4, 1, 1024)), residual.to(DEV), weight.to(DEV), 1e-6)
    e_out, e_sum = opw.add_rms_norm(partial.reshape(3, 4, 1, 1024), residual, weight, 1e-6)
    assert torch.equal(summed.cpu(), e_sum)
    assert (out.cpu() == e_out).float().mean() >= 0.999


def test_swiglu_matches_reference():
    from kernels.swiglu import swiglu
    fx = load("pointwise")
    for case in cases.SWIGLU_CASES:
        packed = cases.swiglu_inputs(case)
        got = swiglu(packed.to(DEV)).cpu()
        assert (got == fx[case[0]]["out"]).float().mean() >= 0.999
        torch.testing.assert_close(got.float(), fx[case[0]]["out"].float(), atol=0.015625, rtol=0.008)


def test_linear_matches_reference():
    """Every epilogue against the reference's projection contract (F.linear, verify_gpu.py:175-185)
    for several split counts: bf16 and fp32 finished tiles (splits summed by a thread-block
    cluster), fp32 split partials; deterministic; finished tiles equal the split-order sum of
    the partials."""
    from kernels import linear as klin
    from kernels._native import lib, ptr, stream, check
    fx = load("pointwise")
    for case in cases.LINEAR_CASES:
        x, weight = cases.linear_inputs(case)
        xd, wd = x.to(DEV), weight.to(DEV)
        got = klin.linear(xd, wd).cpu()
        torch.testing.assert_close(got.float(), fx[case[0]]["out"].float(), atol=1e-3, rtol=0.016)
        assert torch.equal(got, klin.linear(xd, wd).cpu())
        m, k = x.shape
        n = weight.shape[0]
        exact = x.float() @ weight.float().T
        chunks = (k + 63) // 64
        for splits in sorted({1, 2, min(chunks, 7), min(chunks, 8), min(chunks, 12), min(chunks, 16),
                              int(lib.fb_linear_splits(m, n, k)), int(lib.fb_linear_finished_splits(m, n, k)),
                              chunks}):
            _check_finished_splits(xd, wd, exact, splits)


def _check_finished_splits(xd, wd, exact, splits):
    """Split partials sum to the exact product; a finished fp32 tile over the same splits (summed
    by the tile's cluster) equals their split-order sum bit for bit, twice in a row."""
    from kernels._native import lib, ptr, stream, check
    m, k = xd.shape
    n = wd.shape[0]
    part = torch.empty(splits, m, n, dtype=torch.float32, device=DEV)
    check(lib.fb_linear(ptr(xd), ptr(wd), ptr(part), m, n, k, 3, splits, stream()), "fb_linear")
    torch.cuda.synchronize()
    torch.testing.assert_close(part.sum(0).cpu(), exact, atol=1e-4, rtol=1e-4)
    ordered = part[0].clone()
    for s in range(1, splits):
        ordered += part[s]
    for _ in range(2):
        out = torch.empty(m, n, dtype=torch.float32, device=DEV)
        status = lib.fb_linear(ptr(xd), ptr(wd), ptr(out), m, n, k, 1, splits, stream())
        if splits > 8:
            assert status == -2  # a finished tile's splits form one cluster of at most 8 CTAs
            return
        check(status, "fb_linear")
        torch.cuda.synchronize()
        assert torch.equal(out, ordered)  # split-order sum through the cluster


def test_linear_finished_tiles_large_shape():
    """A wide projection (64 rows x 512 tiles) sums its splits through the thread-block cluster
    of each tile: the split-order bits."""
    g = torch.Generator().manual_seed(5)
    x = torch.randn(64, 256, generator=g).bfloat16()
    w = (torch.randn(65536, 256, generator=g) * 0.05).bfloat16()
    exact = x.float() @ w.float().T
    for splits in (2, 4):
        _check_finished_splits(x.to(DEV), w.to(DEV), exact, splits)


def test_linear_split_result_feeds_consumers():
    from kernels.linear import linear
    from kernels.merged import Split
    x = torch.randn(16, 1, 4096, device=DEV).bfloat16()
    w = (torch.randn(1024, 4096, device=DEV) * 0.02).bfloat16()
    res = linear(x, w, split_ok=True)
    expect = torch.nn.functional.linear(x.float(), w.float())
    total = res.partial.sum(0).view(16, 1, 1024) if isinstance(res, Split) else res.float()
    torch.testing.assert_close(total, expect, atol=1e-3, rtol=0.016)


def test_swiglu_linear_matches_oracle():
    """Projection + SwiGLU on 64-row gate/up blocks equals projecting gate and up separately and
    applying the reference's SwiGLU (swiglu.py:13-24), in every form: the split-partials path
    with fb_swiglu_blocked (what swiglu_linear runs when the projection has K splits) and the
    fused epilogue at one split and over K splits summed by the tile's cluster; the split forms
    agree bit for bit."""
    import qwen3
    from kernels import linear as klin
    g = torch.Generator().manual_seed(11)
    for rows, width, hidden in ((1, 3072, 1024), (16, 1536, 4096), (5, 256, 256), (33, 512, 1024), (16, 12288, 4096)):
        x = torch.randn(rows, hidden, generator=g).bfloat16()
        gate = (torch.randn(width, hidden, generator=g) * 0.05).bfloat16()
        up = (torch.randn(width, hidden, generator=g) * 0.05).bfloat16()
        blocked = qwen3.interleave_gate_up(gate, up).contiguous().to(DEV)
        expect = opw.swiglu(torch.cat((opw.linear(x, gate), opw.linear(x, up)), -1))
        xd = x.to(DEV)
        forms = {"swiglu_linear": klin.swiglu_linear(xd, blocked)}
        chunks = hidden // 64
        for splits in sorted({1, 2, min(chunks, 4), min(chunks, 8)}):
            forms[f"epilogue S={splits}"] = klin.project(xd, blocked, klin.SWIGLU_OUT, splits)
        splits = klin.splits_for(rows, 2 * width, hidden, xd.device)
        if splits > 1:
            partials = klin.project(xd, blocked, klin.SPLITS_OUT, splits)
            out = torch.empty(rows, width, dtype=torch.bfloat16, device=DEV)
            from kernels._native import check, lib, ptr, stream
            check(lib.fb_swiglu_blocked(ptr(partials), splits, ptr(out), rows, width, stream()), "fb_swiglu_blocked")
            forms["split consumer"] = out
            if splits <= 8:
                assert torch.equal(out, forms.get(f"epilogue S={splits}", klin.project(xd, blocked, klin.SWIGLU_OUT,
                                                                                       splits)))
        for name, got in forms.items():
            got = got.cpu()
            assert (got == expect).float().mean() >= 0.99, name
            torch.testing.assert_close(got.float(), expect.float(), atol=0.015625, rtol=0.016, msg=name)


def test_argmax_matches_reference():
    from kernels.argmax import argmax
    fx = load("pointwise")
    for case in cases.ARGMAX_CASES:
        logits = cases.argmax_inputs(case)
        top = torch.zeros(logits.shape[0], dtype=torch.float32, device=DEV)
        ids = argmax(logits.to(DEV), top=top).cpu()
        assert torch.equal(ids, fx[case[0]]["out"])
        assert torch.equal(top.cpu(), fx[case[0]]["top"])


def test_fused_argmax_equals_projection_then_argmax():
    """fb_linear_argmax + fb_argmax_candidates (logits never written) give torch.argmax of the
    bf16 logits the one-split projection stores, ties to the lowest index, for ragged vocab
    tails, planted ties, -inf rows and a vocabulary offset (engine/kernels/argmax.py:73-129)."""
    from kernels import linear as klin
    from kernels.argmax import fused_argmax, greedy_tokens
    g = torch.Generator().manual_seed(11)
    for rows, n, k in ((1, 151936, 1024), (16, 18992, 4096), (5, 1000, 256), (33, 4104, 512), (64, 136, 64)):
        x = torch.randn(rows, k, generator=g).bfloat16().to(DEV)
        w = (torch.randn(n, k, generator=g) * 0.05).bfloat16().to(DEV)
        if n == 136:
            w[7] = w[130]  # identical rows: identical logits, the lower index must win
        logits = klin.project(x, w, klin.BF16_OUT, 1)
        expect = torch.argmax(logits.float(), dim=-1)
        got = fused_argmax(x, w)
        assert torch.equal(got, expect), (rows, n, k)
        assert torch.equal(fused_argmax(x, w, index_base=1000), expect + 1000)
        assert torch.equal(greedy_tokens(x, w, klin.linear), expect)
        ids, full = greedy_tokens(x, w, klin.linear, top=torch.zeros(rows, device=DEV))
        assert full.shape == (rows, n)
    # a row whose logits are all -inf picks index 0, as torch.argmax does
    x = torch.zeros(2, 64, device=DEV).bfloat16()
    x[1, 0] = float("-inf")
    w = torch.ones(256, 64, device=DEV).bfloat16()
    assert fused_argmax(x, w).tolist() == torch.argmax(klin.project(x, w, klin.BF16_OUT, 1).float(), -1).tolist()


def test_decode_attention_fused_equals_two_launch_and_counters_reset():
    """fb_decode_attention (persistent form, last CTA merges) equals fb_decode_attention_partials
    + fb_decode_attention_combine bit for bit, and leaves its per-pair counters at zero. Per-row
    positions (two or more rows) keep every call on the persistent form."""
    from kernels.decode_attention import _ctas, attend, workspace_bytes
    for lengths, q_heads in (([1, 700, 8192, 65], 32), ([30000, 20001], 16), ([300, 301, 302, 303, 1, 2, 3, 4], 16)):
        q, k, v, position = _ragged(len(lengths), q_heads, 8, 128, lengths, seed=sum(lengths))
        ctas = _ctas((q.device, len(lengths), 8, k.shape[2], 128))
        ws = torch.zeros(workspace_bytes(len(lengths), q_heads, 8, 128, ctas), dtype=torch.uint8, device=DEV)
        fused = attend(q, k, v, position, 0.088, workspace=ws.clone(), ctas=ctas)
        again_ws = torch.zeros_like(ws)
        attend(q, k, v, position, 0.088, workspace=again_ws, ctas=ctas)
        second = attend(q, k, v, position, 0.088, workspace=again_ws, ctas=ctas)  # reuses the counters
        two = attend(q, k, v, position, 0.088, workspace=ws.clone(), ctas=ctas, two_launch=True)
        torch.cuda.synchronize()
        assert torch.equal(fused, two)
        assert torch.equal(second, fused)
        counters = again_ws[-len(lengths) * 8 * 4:].view(torch.int32)
        assert int(counters.abs().sum()) == 0


def test_allreduce_single_rank():
    """The TP all-reduce at world 1 (every region is this GPU's own): fb_reduce_scatter_push stores
    the split-order sum of the projection's K-split partials as flagged fp32 words; the owner
    phase of fb_allreduce_add_rmsnorm then writes the summed bf16 pairs and the row's sum of
    squares, flagged, and the result equals add_rms_norm over the same partials (the residual sum
    bit for bit, the normalized row within the norm's reduction-order ULPs)."""
    import ctypes
    from kernels import linear as klin
    from kernels._native import lib, ptr, stream, check
    from kernels.merged import Split
    from kernels.rmsnorm import add_rms_norm
    g = torch.Generator().manual_seed(21)
    m, n, k = 16, 4096, 1536
    x = torch.randn(m, k, generator=g).bfloat16().to(DEV)
    w = (torch.randn(n, k, generator=g) * 0.05).bfloat16().to(DEV)
    residual = torch.randn(m, n, generator=g).bfloat16().to(DEV)
    gain = torch.randn(n, generator=g).bfloat16().to(DEV)
    epoch = torch.full((1,), 9, dtype=torch.int64, device=DEV)
    exact = x.float() @ w.float().T
    splits = int(lib.fb_linear_splits(m, n, k))
    assert splits > 1
    part = klin.project(x, w, klin.SPLITS_OUT, splits)
    ordered = part[0].clone()
    for s in range(1, splits):
        ordered += part[s]
    rs = torch.zeros(2, 1, m, n, dtype=torch.int64, device=DEV)  # two uses
    ag = torch.zeros(2, m, n // 2, dtype=torch.int64, device=DEV)
    ss = torch.zeros(2, 1, n // 512, m, dtype=torch.int64, device=DEV)  # [uses, world, slice chunks, rows]
    use = 1
    check(lib.fb_reduce_scatter_push(ptr(part), splits, m, n, 1, 0, use, (ctypes.c_void_p * 1)(rs.data_ptr()),
                                     ptr(epoch), stream()), "fb_reduce_scatter_push")
    out, summed = torch.empty_like(residual), torch.empty_like(residual)
    check(lib.fb_allreduce_add_rmsnorm(ptr(rs), ptr(ag), ptr(ss), (ctypes.c_void_p * 1)(ag.data_ptr()),
                                       (ctypes.c_void_p * 1)(ss.data_ptr()), use, 1, 0, ptr(epoch), ptr(residual),
                                       ptr(gain), ptr(out), ptr(summed), m, n, 1e-6, stream()),
          "fb_allreduce_add_rmsnorm")
    torch.cuda.synchronize()
    halves = rs[use].view(torch.int32).view(m, n, 2)  # little-endian: [value bits, flag]
    assert bool((halves[..., 1] == 10).all())
    words = halves[..., 0].contiguous().view(torch.float32)
    torch.testing.assert_close(words, exact, atol=1e-4, rtol=1e-4)
    assert torch.equal(words, ordered)
    assert bool((rs[0] == 0).all()) and bool((ag[0] == 0).all())  # use 0 untouched
    assert bool((ag[use].view(torch.int32).view(m, n // 2, 2)[..., 1] == 10).all())
    e_out, e_sum = add_rms_norm(Split(part, (m, n)), residual, gain, 1e-6)
    assert torch.equal(summed, e_sum)
    assert (out == e_out).float().mean() >= 0.999 and ulps(out, e_out).max() <= 2


def test_allreduce_push_single_rank():
    """The push-form TP all-reduce at world 1: fb_allreduce_push stores the split-order sum of the
    projection's K-split partials as flagged fp32 words (flag = epoch + 1 in the high half) into
    slab `rank` of recv[use]; fb_allreduce_sum_add_rmsnorm then equals add_rms_norm over the same
    partials (the residual sum bit for bit, the normalized row within the norm's ULPs)."""
    import ctypes
    from kernels import linear as klin
    from kernels._native import lib, ptr, stream, check
    from kernels.merged import Split
    from kernels.rmsnorm import add_rms_norm
    g = torch.Generator().manual_seed(22)
    m, n, k = 16, 4096, 1536
    x = torch.randn(m, k, generator=g).bfloat16().to(DEV)
    w = (torch.randn(n, k, generator=g) * 0.05).bfloat16().to(DEV)
    residual = torch.randn(m, n, generator=g).bfloat16().to(DEV)
    gain = torch.randn(n, generator=g).bfloat16().to(DEV)
    epoch = torch.full((1,), 12, dtype=torch.int64, device=DEV)
    splits = int(lib.fb_linear_splits(m, n, k))
    part = klin.project(x, w, klin.SPLITS_OUT, splits)
    ordered = part[0].clone()
    for s_ in range(1, splits):
        ordered += part[s_]
    recv = torch.zeros(2, 1, m, n, dtype=torch.int64, device=DEV)  # two uses, world 1
    use = 1
    check(lib.fb_allreduce_push(ptr(part), splits, m, n, 1, 0, use, (ctypes.c_void_p * 1)(recv.data_ptr()),
                                ptr(epoch), stream()), "fb_allreduce_push")
    out, summed = torch.empty_like(residual), torch.empty_like(residual)
    check(lib.fb_allreduce_sum_add_rmsnorm(ptr(recv), use, 1, ptr(epoch), ptr(residual), ptr(gain), ptr(out),
                                           ptr(summed), m, n, 1e-6, stream()), "fb_allreduce_sum_add_rmsnorm")
    torch.cuda.synchronize()
    halves = recv[use, 0].view(torch.int32).view(m, n, 2)  # little-endian: [value bits, flag]
    assert bool((halves[..., 1] == 13).all())
    assert torch.equal(halves[..., 0].contiguous().view(torch.float32), ordered)
    assert bool((recv[0] == 0).all())  # use 0 untouched
    e_out, e_sum = add_rms_norm(Split(part, (m, n)), residual, gain, 1e-6)
    assert torch.equal(summed, e_sum)
    assert (out == e_out).float().mean() >= 0.999 and ulps(out, e_out).max() <= 2


@pytest.mark.parametrize("splits", [0, 6, 16])
def test_qk_rope_cache_bit_exact_at_config4_shapes(splits):
    """The decode-step K cache append at the Qwen3-8B shapes (batch 16, 32/8 heads, D 128, one
    shared position in an 8200-slot cache, whole RoPE tables) against the oracle, bit for bit: K,
    V and Q, from bf16 input and from fp32 split-K partials (6 is the TP1 qkv projection's split
    count, 16 the TP8 shard's)."""
    g = torch.Generator().manual_seed(100 + splits)
    batch, hq, hkv, dim, capacity = 16, 32, 8, 128, 8200
    width = (hq + 2 * hkv) * dim
    if splits == 0:
        packed = (torch.randn(batch, 1, width, generator=g) * 3).bfloat16()
    else:
        packed = torch.randn(splits, batch, width, generator=g) * 0.7
    q_gain = (1 + 0.1 * torch.randn(dim, generator=g)).bfloat16()
    k_gain = (1 + 0.1 * torch.randn(dim, generator=g)).bfloat16()
    keys = torch.randn(batch, hkv, capacity, dim, generator=g).bfloat16()
    values = torch.randn(batch, hkv, capacity, dim, generator=g).bfloat16()
    position = torch.tensor([8191], dtype=torch.int64)
    inv = 1.0 / (1e6 ** (torch.arange(0, dim, 2).float() / dim))
    angle = torch.arange(capacity).float()[:, None] * inv[None, :]
    angle = torch.cat((angle, angle), -1)
    cos, sin = angle.cos().bfloat16(), angle.sin().bfloat16()
    ok, ov = keys.clone(), values.clone()
    expect_q = opw.qk_rope_cache(packed, q_gain, k_gain, 1e-6, 1e-6, cos, sin, position, ok, ov, hq,
                                 rows=False, phases=torch.zeros(batch, 1, dtype=torch.int64))
    from kernels._native import check, lib, ptr, stream
    # device copies held in names until the kernel has run (a temporary's memory could be reused)
    kd, vd, pd = keys.to(DEV), values.to(DEV), packed.to(DEV)
    qg, kg, cd, sd, posd = q_gain.to(DEV), k_gain.to(DEV), cos.to(DEV), sin.to(DEV), position.to(DEV)
    query = torch.empty(batch, 1, hq, dim, dtype=torch.bfloat16, device=DEV)
    # the decode step's call: mode 0 (one shared position), whole cos/sin tables
    check(lib.fb_qk_norm_rope_append(ptr(pd), splits, ptr(qg), ptr(kg), 1e-6, 1e-6, ptr(cd), ptr(sd), ptr(posd),
                                     None, ptr(query), ptr(kd), ptr(vd), batch, 1, hq, hkv, dim, capacity, 0, 1,
                                     stream()), "fb_qk_norm_rope_append")
    torch.cuda.synchronize()
    got_q = query.cpu()
    for name, got, want in (("keys", kd.cpu(), ok), ("values", vd.cpu(), ov), ("query", got_q, expect_q)):
        differ = (got != want).nonzero()
        assert differ.numel() == 0, f"{name}: {differ.shape[0]} elements differ, first {differ[:4].tolist()}"
