"""Oracle: norms, RoPE/KV append, SwiGLU, projections, argmax (CPU, TEST INFRASTRUCTURE ONLY).

Restates, with the reference's bf16 cast points, in fp32 torch on the CPU:
  engine/kernels/rmsnorm.py:21-46    `_rms_norm_kernel`        (references.py:42-49)
  engine/kernels/rmsnorm.py:75-95    `_add_rms_norm_kernel`    (references.py:52-64)
  engine/kernels/rmsnorm.py:128-142  `_embed_rms_norm_kernel`  (references.py:120-130)
  engine/kernels/swiglu.py:13-24     `_swiglu`                 (references.py:133-140)
  engine/kernels/qk_rope.py:13-84    `_qk_rope_cache`          (references.py:143-192)
  engine/kernels/merged.py:37-45     `load_merged`             (references.py:30-39)
  engine/kernels/linear.py:27-93     projections: fp32 accumulation, one bf16 rounding
  engine/kernels/argmax.py:19-48     first-index argmax        (references.py:67-87)
"""

import torch

BF16, F32 = torch.bfloat16, torch.float32


def merged(partial):
    """merged.py:37-45: fp32 partials [S, ...] summed in split order, rounded to bf16."""
    total = partial[0].clone()
    for split in range(1, partial.shape[0]):
        total += partial[split]
    return total.to(BF16)


def rms_norm(x, weight, eps):
    """rmsnorm.py:35-46: y = bf16(bf16(x * rsqrt(mean(x^2) + eps)) * w)."""
    xf = x.to(F32)
    normed = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return normed.to(BF16) * weight


def add_rms_norm(x, residual, weight, eps):
    """rmsnorm.py:75-95: sum = bf16(x + r); out = bf16(bf16(sum * rsqrt(...)) * w). ``x`` may be
    fp32 split partials [S, ..., W] (summed and rounded first)."""
    if x.dtype == F32:
        x = merged(x).reshape(residual.shape)
    summed = (x.to(F32) + residual.to(F32)).to(BF16)
    s32 = summed.to(F32)
    variance = s32.pow(2).mean(-1, keepdim=True)
    normalized = (s32 * torch.rsqrt(variance + eps)).to(BF16).to(F32)
    return (normalized * weight.to(F32)).to(BF16), summed


def embed_rms_norm(token_ids, table, weight, eps):
    """rmsnorm.py:128-142: hidden = table[ids]; y = rms_norm(hidden)."""
    hidden = table[token_ids.reshape(-1)].reshape(*token_ids.shape, table.shape[1])
    return rms_norm(hidden, weight, eps), hidden


def swiglu(packed):
    """swiglu.py:13-24: bf16(bf16(g / (1 + exp(-g))) * u) from [.., 2I] = [gate | up]."""
    if packed.dtype == F32:
        packed = merged(packed)
    data = packed.to(F32)
    width = data.shape[-1] // 2
    gate, up = data[..., :width], data[..., width:]
    activated = (gate / (1.0 + torch.exp(-gate))).to(BF16).to(F32)
    return (activated * up).to(BF16)


def linear(x, weight):
    """x @ W^T with fp32 accumulation and one bf16 rounding (linear.py:1-6 contract)."""
    return (x.to(F32) @ weight.to(F32).T).to(BF16)


def argmax(logits):
    """argmax.py:1-9: first index of the row maximum (bf16 -> fp32 exact)."""
    return logits.to(F32).argmax(-1)


def sum_squares_host_order(x):
    """Sum of squares over the last dim (a multiple of 32) in the order torch's CPU sum kernel
    adds a contiguous fp32 row: 8-wide vectors, four interleaved vector accumulators
    (a_k = v_k + v_{k+4} + ... in order), then ((a_0 + a_1) + a_2) + a_3, then the 8 lanes in
    order. That is what the reference's eager ``x.pow(2).mean(-1)`` computes in the fixtures
    (references.py:155); written out with elementwise adds so the answer does not depend on the
    host's vector width."""
    dim = x.shape[-1]
    assert dim % 32 == 0
    vectors = (x * x).reshape(*x.shape[:-1], dim // 8, 8)
    acc = [vectors[..., k, :].clone() for k in range(4)]
    for r in range(1, dim // 32):
        for k in range(4):
            acc[k] = acc[k] + vectors[..., 4 * r + k, :]
    vec = ((acc[0] + acc[1]) + acc[2]) + acc[3]
    total = vec[..., 0].clone()
    for lane in range(1, 8):
        total = total + vec[..., lane]
    return total


def qk_rope_cache(packed, q_weight, k_weight, q_eps, k_eps, cos, sin, position, keys, values,
                  q_heads, prefill=False, rows=False, phases=None):
    """qk_rope.py:13-84 / references.py:143-192.

    packed bf16 [B, T, (Hq + 2Hkv) D] (or fp32 partials [S, B*T, ...]); keys/values
    [B, Hkv, C, D] are modified in place; returns token-major Q [B, T, Hq, D].
    """
    batch, kv_heads, capacity, dim = keys.shape
    if packed.dtype == F32:
        tokens = packed.shape[1] // batch
        data = merged(packed).reshape(batch * tokens, q_heads + 2 * kv_heads, dim)
    else:
        tokens = packed.shape[1]
        data = packed.reshape(batch * tokens, q_heads + 2 * kv_heads, dim)
    heads = q_heads + kv_heads
    x = data[:, :heads].to(F32)
    eps = torch.cat((torch.full((q_heads,), q_eps), torch.full((kv_heads,), k_eps)))[None, :, None]
    mean = (sum_squares_host_order(x) / dim)[..., None]
    inv_std = torch.rsqrt(mean + eps)
    gain = torch.cat((q_weight.to(F32).expand(q_heads, dim), k_weight.to(F32).expand(kv_heads, dim)))[None]
    normalized = (x * inv_std).to(BF16).to(F32)
    weighted = (normalized * gain).to(BF16).to(F32)
    half = dim // 2
    rotated = torch.cat((-weighted[..., half:], weighted[..., :half]), dim=-1)
    pos = position.reshape(-1).to(torch.int64)
    if phases is not None:
        offsets = pos.repeat_interleave(tokens) + phases.reshape(-1).to(torch.int64)
        cosine = cos.reshape(-1, dim).to(F32)[offsets]
        sine = sin.reshape(-1, dim).to(F32)[offsets]
    else:
        count = batch * tokens if rows else tokens
        cosine = cos.reshape(count, dim).to(F32)
        sine = sin.reshape(count, dim).to(F32)
        if not rows:
            cosine, sine = cosine.repeat(batch, 1), sine.repeat(batch, 1)
    direct = (weighted * cosine[:, None, :]).to(BF16).to(F32)
    turn = (rotated * sine[:, None, :]).to(BF16).to(F32)
    result = (direct + turn).to(BF16)
    query = result[:, :q_heads].reshape(batch, tokens, q_heads, dim).clone()
    new_keys = result[:, q_heads:].reshape(batch, tokens, kv_heads, dim)
    new_values = data[:, heads:].reshape(batch, tokens, kv_heads, dim)
    for b in range(batch):
        for t in range(tokens):
            slot = t if prefill else int(pos[b if rows else 0]) + t
            assert 0 <= slot < capacity
            keys[b, :, slot] = new_keys[b, t]
            values[b, :, slot] = new_values[b, t]
    return query
