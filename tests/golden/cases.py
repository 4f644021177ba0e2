"""Seeded input builders for the golden fixtures (shared by make_golden.py and the tests).

Inputs are regenerated from seeds rather than stored; each fixture records the SHA-256
of the inputs it was made from, so a test first proves it rebuilt the same bytes.
Shapes come from the reference's own checks (agent/verify_gpu.py:98-173,
agent/local_cpu/check_block_attention.py:65-73) and from BASELINE.json's configs.
"""

import hashlib
import math

import torch

BF16 = torch.bfloat16


def digest(*tensors):
    h = hashlib.sha256()
    for t in tensors:
        if t is None:
            continue
        t = t.contiguous()
        h.update(str(tuple(t.shape)).encode())
        h.update(str(t.dtype).encode())
        h.update(t.view(torch.uint8).numpy().tobytes() if t.dtype != torch.bool else t.numpy().tobytes())
    return h.hexdigest()


def _gen(seed):
    return torch.Generator().manual_seed(seed)


# ---------------------------------------------------------------- decode attention
# (name, batch, q_heads, kv_heads, dim, capacity, positions, magnitude, seed, nan_tail)
DECODE_CASES = [
    # B=1, 16/8 heads, D=128, L=2048, seed 0 (Q, K, V order), 8 splits.
    ("c1", 1, 16, 8, 128, 2048, [2047], 1.0, 0, False),
    # agent/verify_gpu.py:154-158 shapes (B, Hkv, D, C, valid), Hq = 4 Hkv, magnitudes 1 and 3,
    # unused slots poisoned with NaN (:165-168).
    ("v1", 1, 32, 8, 128, 1, [0], 1.0, 11, True),
    ("v2", 1, 32, 8, 128, 65, [0], 1.0, 12, True),
    ("v3", 1, 32, 8, 128, 65, [32], 3.0, 13, True),
    ("v4", 1, 32, 8, 128, 544, [512], 1.0, 14, True),
    ("v5", 4, 32, 8, 128, 2080, [2047], 3.0, 15, True),
    ("v6", 16, 32, 8, 128, 640, [638], 1.0, 16, True),
    ("v7", 2, 8, 2, 64, 65, [64], 3.0, 17, True),
    # ragged rows (per-row positions), the BASELINE config-3 head shape at small lengths
    ("r1", 4, 32, 8, 128, 3000, [1023, 2999, 1500, 0], 1.0, 21, True),
    ("r2", 3, 16, 8, 64, 300, [299, 63, 64], 1.0, 22, True),
]


def decode_inputs(case):
    name, batch, q_heads, kv_heads, dim, capacity, positions, magnitude, seed, nan_tail = case
    g = _gen(seed)
    q = (torch.randn(batch, q_heads, 1, dim, generator=g) * magnitude).to(BF16)
    k = (torch.randn(batch, kv_heads, capacity, dim, generator=g) * magnitude).to(BF16)
    v = torch.randn(batch, kv_heads, capacity, dim, generator=g).to(BF16)
    position = torch.tensor(positions, dtype=torch.int64)
    if nan_tail:
        for b in range(batch):
            valid = int(positions[b if len(positions) > 1 else 0]) + 1
            k[b, :, valid:] = float("nan")
            v[b, :, valid:] = float("nan")
    scale = 1.0 / math.sqrt(dim)
    return q, k, v, position, scale


# ---------------------------------------------------------------- verify (block) attention
# (name, batch, tokens, q_heads, kv_heads, dim, capacity, positions, chains, splits, seed)
BLOCK_CASES = [
    # B=8, T=5, 32/8 heads, D=128, 4096 prefix + 5 new slots, chain 5.
    ("c5", 8, 5, 32, 8, 128, 4101, [4096] * 8, [5] * 8, 1, 0),
    # check_block_attention.py:65-73 style: chains T, T-2, 2, 1; position 0; several splits.
    ("b1", 2, 5, 8, 2, 128, 200, [150, 0], [5, 3], 1, 31),
    ("b2", 3, 4, 16, 4, 64, 130, [100, 20, 125], [2, 1, 4], 3, 32),
    ("b3", 2, 8, 32, 8, 128, 520, [511, 300], [8, 6], 4, 33),
]


def block_inputs(case):
    name, batch, tokens, q_heads, kv_heads, dim, capacity, positions, chains, splits, seed = case
    g = _gen(seed)
    q = torch.randn(batch, tokens, q_heads, dim, generator=g).to(BF16)
    k = torch.randn(batch, kv_heads, capacity, dim, generator=g).to(BF16)
    v = torch.randn(batch, kv_heads, capacity, dim, generator=g).to(BF16)
    position = torch.tensor(positions, dtype=torch.int64)
    chain = torch.tensor(chains, dtype=torch.int64)
    # Junk past each row's block: never visible (check_block_attention.py:67-69 uses 1e6 tails).
    for b in range(batch):
        end = positions[b] + tokens
        k[b, :, end:] = 1e6
        v[b, :, end:] = 1e6
    return q, k, v, position, chain, 1.0 / math.sqrt(dim), splits


# ---------------------------------------------------------------- QK norm + RoPE + append
# (name, batch, tokens, q_heads, kv_heads, dim, capacity, mode, splits, seed)
# mode: "decode" (position [1]), "prefill" (slots 0..T-1), "rows" (position [B]), "table"
ROPE_CASES = [
    ("q1", 1, 1, 32, 8, 128, 9, "decode", 1, 41),   # verify_gpu.py:98 shapes
    ("q2", 4, 1, 32, 8, 128, 9, "decode", 1, 42),
    ("q3", 2, 1, 8, 2, 64, 9, "decode", 1, 43),
    ("q4", 2, 1, 32, 8, 128, 12, "decode", 3, 44),  # split-K fp32 input
    ("q5", 2, 6, 16, 8, 128, 10, "prefill", 1, 45),
    ("q6", 3, 4, 32, 8, 128, 40, "rows", 1, 46),
    ("q7", 2, 5, 32, 8, 128, 64, "table", 2, 47),
]


def rope_inputs(case):
    name, batch, tokens, q_heads, kv_heads, dim, capacity, mode, splits, seed = case
    g = _gen(seed)
    width = (q_heads + 2 * kv_heads) * dim
    if splits == 1:
        packed = torch.randn(batch, tokens, width, generator=g).to(BF16)
    else:
        packed = torch.randn(splits, batch * tokens, width, generator=g) * 0.5
    q_weight = torch.randn(dim, generator=g).to(BF16)
    k_weight = torch.randn(dim, generator=g).to(BF16)
    q_eps, k_eps = 1e-6, 1e-3
    keys = torch.full((batch, kv_heads, capacity, dim), 17.0).to(BF16)
    values = torch.full((batch, kv_heads, capacity, dim), -13.0).to(BF16)
    phases = None
    if mode == "table":
        angle = torch.arange(capacity, dtype=torch.float32)[:, None] * torch.rand(dim // 2, generator=g)[None, :]
        angle = torch.cat((angle, angle), dim=-1)
        cos, sin = angle.cos().to(BF16), angle.sin().to(BF16)
        position = torch.randint(0, capacity - tokens, (batch,), generator=g)
        phases = torch.tensor([[0, 1, 2, 1, 1][:tokens]] * batch, dtype=torch.int64)
    else:
        count = batch * tokens if mode == "rows" else tokens
        phase = torch.randn(count, dim // 2, generator=g)
        phase = torch.cat((phase, phase), dim=-1)
        cos, sin = phase.cos().to(BF16), phase.sin().to(BF16)
        if mode == "decode":
            position = torch.tensor([3 if capacity > 4 else 0], dtype=torch.int64)
        elif mode == "prefill":
            position = torch.arange(tokens, dtype=torch.int64)
        else:
            position = torch.randint(0, capacity - tokens, (batch,), generator=g)
    return dict(packed=packed, q_weight=q_weight, k_weight=k_weight, q_eps=q_eps, k_eps=k_eps, cos=cos,
                sin=sin, position=position, keys=keys, values=values, q_heads=q_heads,
                prefill=mode == "prefill", rows=mode in ("rows", "table"), phases=phases)


# ---------------------------------------------------------------- pointwise kernels
NORM_CASES = [("n1", 1, 1024, 51), ("n2", 16, 4096, 52), ("n3", 31, 256, 53), ("n4", 9, 128, 54), ("n5", 2, 2560, 55)]
SWIGLU_CASES = [("s1", 1, 9728, 61), ("s2", 16, 9728, 62), ("s3", 19, 512, 63), ("s4", 4, 3072, 64)]
LINEAR_CASES = [("l1", 1, 256, 512, 71), ("l2", 4, 512, 1024, 72), ("l3", 16, 1024, 4096, 73),
                ("l4", 1, 6144, 2560, 74), ("l5", 33, 384, 640, 75), ("l6", 5, 2048, 3072, 76)]
ARGMAX_CASES = [("a1", 1, 151936, 81), ("a2", 16, 151936, 82), ("a3", 3, 1000, 83)]


def norm_inputs(case):
    name, rows, width, seed = case
    g = _gen(seed)
    x = torch.randn(rows, width, generator=g).to(BF16)
    residual = torch.randn(rows, width, generator=g).to(BF16)
    weight = torch.randn(width, generator=g).to(BF16)
    table = torch.randn(97, width, generator=g).to(BF16)
    ids = torch.randint(0, 97, (rows,), generator=g)
    return x, residual, weight, 1e-6, table, ids


def swiglu_inputs(case):
    name, rows, width, seed = case
    g = _gen(seed)
    packed = torch.randn(rows, 2 * width, generator=g).to(BF16)
    packed[:, :8] = torch.tensor([-100, -20, -1, 0, 1, 20, 100, 0.125]).to(BF16)  # verify_gpu.py:87-89
    return packed


def linear_inputs(case):
    name, rows, outputs, width, seed = case
    g = _gen(seed)
    x = torch.randn(rows, width, generator=g).to(BF16)
    weight = (torch.randn(outputs, width, generator=g) * 0.02).to(BF16)
    return x, weight


def argmax_inputs(case):
    name, rows, vocab, seed = case
    g = _gen(seed)
    logits = torch.randn(rows, vocab, generator=g).to(BF16)
    # planted ties: the lowest index must win
    for r in range(rows):
        best = float(logits[r].float().max()) + 1.0
        a, b = int(torch.randint(0, vocab, (1,), generator=g)), int(torch.randint(0, vocab, (1,), generator=g))
        logits[r, max(a, b)] = best
        logits[r, min(a, b)] = best
    return logits


# ---------------------------------------------------------------- tiny Qwen3 (agent/verify_gpu.py:195-201)
TINY_QWEN3 = dict(vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                  num_attention_heads=8, num_key_value_heads=2, head_dim=64, max_position_embeddings=4096,
                  rope_theta=5_000_000.0, tie_word_embeddings=True, rms_norm_eps=1e-6)
MODEL_CASES = [("m1", 1, 7, 6, 91), ("m2", 3, 13, 5, 92)]  # (name, batch, prompt, new tokens, seed)


def tiny_qwen3_weights(seed=90):
    """Random tiny-Qwen3 weights (linear ~N(0, 0.02), norms ~1 + N(0, 0.1)), keyed by HF names."""
    cfg = TINY_QWEN3
    g = _gen(seed)
    h, i, d = cfg["hidden_size"], cfg["intermediate_size"], cfg["head_dim"]
    hq, hkv = cfg["num_attention_heads"], cfg["num_key_value_heads"]

    def lin(o, n):
        return (torch.randn(o, n, generator=g) * 0.08).to(BF16)

    def norm(n):
        return (1.0 + 0.1 * torch.randn(n, generator=g)).to(BF16)

    w = {"model.embed_tokens.weight": (torch.randn(cfg["vocab_size"], h, generator=g) * 0.25).to(BF16),
         "model.norm.weight": norm(h)}
    for layer in range(cfg["num_hidden_layers"]):
        p = f"model.layers.{layer}."
        w[p + "input_layernorm.weight"] = norm(h)
        w[p + "post_attention_layernorm.weight"] = norm(h)
        w[p + "self_attn.q_proj.weight"] = lin(hq * d, h)
        w[p + "self_attn.k_proj.weight"] = lin(hkv * d, h)
        w[p + "self_attn.v_proj.weight"] = lin(hkv * d, h)
        w[p + "self_attn.o_proj.weight"] = lin(h, hq * d)
        w[p + "self_attn.q_norm.weight"] = norm(d)
        w[p + "self_attn.k_norm.weight"] = norm(d)
        w[p + "mlp.gate_proj.weight"] = lin(i, h)
        w[p + "mlp.up_proj.weight"] = lin(i, h)
        w[p + "mlp.down_proj.weight"] = lin(h, i)
    return w


def model_prompt(case):
    name, batch, prompt, steps, seed = case
    return torch.randint(3, TINY_QWEN3["vocab_size"], (batch, prompt), generator=_gen(seed)), steps


# ---------------------------------------------------------------- speculation bookkeeping
# (name, batch, size, tokens per row, drafts by match length, successor width, vocab, seed)
SPEC_CASES = [
    ("p1", 4, 64, 8, (2, 4, 6, 7), 8, 5, 101),       # tiny vocabulary: long suffix matches
    ("p2", 3, 200, 16, (5, 8, 13, 14), 8, 12, 102),
    ("p3", 2, 40, 5, (2, 3, 4, 4), 4, 7, 103),
    ("p4", 5, 300, 2, (1, 1, 1, 1), 8, 30, 104),     # no alternative lanes
    ("p5", 2, 130, 16, (15, 15, 15, 15), 8, 9, 105),  # chain only, no alternatives
    ("p6", 16, 2048, 16, (5, 8, 13, 14), 8, 50, 106),
]


def spec_inputs(case):
    """History, position, successor table, stale hints and a greedy pass for one case.

    Histories repeat short motifs so that suffix matches of every length occur; positions
    leave room for a settle to write TOKENS slots; the greedy tokens agree with a random
    number of chain drafts (planted after propose, see spec_greedy)."""
    name, batch, size, tokens, drafts, top, vocab, seed = case
    g = _gen(seed)
    motif = torch.randint(0, vocab, (max(3, size // 7),), generator=g)
    history = torch.empty(batch, size, dtype=torch.int64)
    for b in range(batch):
        pieces, n = [], 0
        while n < size:
            if torch.rand((), generator=g) < 0.5:
                start = int(torch.randint(0, motif.numel(), (), generator=g))
                piece = motif[start:start + int(torch.randint(1, 9, (), generator=g))]
            else:
                piece = torch.randint(0, vocab, (int(torch.randint(1, 5, (), generator=g)),), generator=g)
            pieces.append(piece)
            n += piece.numel()
        history[b] = torch.cat(pieces)[:size]
    position = torch.randint(0, size - tokens - 1, (batch,), generator=g)
    position[0] = size - tokens - 1  # the latest possible place
    successor = torch.randint(0, vocab, (vocab, top), generator=g)
    stale = torch.randint(-1, vocab, (batch,), generator=g)
    limit = position + torch.randint(0, tokens + 3, (batch,), generator=g)
    return {"history": history, "position": position, "successor": successor, "stale": stale, "limit": limit,
            "tokens": tokens, "drafts": drafts, "vocab": vocab, "seed": seed}


def spec_greedy(proposed, chains, vocab, seed):
    """A verify pass's greedy tokens for proposed rows: each row accepts a random number of
    its chain drafts (greedy[slot] = draft[slot + 1]); some rows put an alternative lane's
    token first (the branch path)."""
    g = _gen(seed + 1000)
    batch, tokens = proposed.shape
    greedy = torch.randint(0, vocab, (batch, tokens), generator=g)
    for b in range(batch):
        chain = int(chains[b])
        keep = int(torch.randint(0, chain, (), generator=g))
        for slot in range(keep):
            greedy[b, slot] = proposed[b, slot + 1]
        if keep == 0 and chain < tokens and torch.rand((), generator=g) < 0.5:
            greedy[b, 0] = proposed[b, int(torch.randint(chain, tokens, (), generator=g))]
    return greedy


def spec_margin_inputs(case, proposed):
    """Logits [B*T, V] (bf16), their per-row maxima as fp32 and a margin for within_margin."""
    name, batch, size, tokens, drafts, top, vocab, seed = case
    g = _gen(seed + 2000)
    logits = (torch.randn(batch * tokens, vocab, generator=g) * 2).bfloat16()
    best = logits.float().max(-1).values
    return logits, best, 0.75


def relocate_inputs(seed=110):
    g = _gen(seed)
    store = torch.randn(2, 3, 4, 2, 40, 64, generator=g).bfloat16()
    move_from = torch.tensor([5, -1, 39, 12], dtype=torch.int64)
    move_to = torch.tensor([3, 7, 30, 13], dtype=torch.int64)
    return store, move_from, move_to
