"""Oracle: decode / verify attention (CPU, TEST INFRASTRUCTURE ONLY).

Restates the reference's split-KV decode attention and its verify (block) attention:
  engine/kernels/decode_attention.py:31-101  `_decode_partials` (interval softmax)
  engine/kernels/decode_attention.py:104-127 `_decode_merge` (log-sum-exp combine)
  engine/kernels/decode_attention.py:152-157 `_default_config` (split policy)
  engine/kernels/decode_attention.py:260-350 `_block_partials` (verify masks :286-292, :323)
  engine/kernels/decode_attention.py:455-478 `_block_merge`
in the form of the reference's own CPU restatement (agent/local_cpu/shim/references.py:
`_interval` :195-205, `_decode_partials` :208-228, `_merge` :231-238, `_block_partials`
:250-285): fp32 scores scaled by scale*log2(e), exp2 softmax per interval, probabilities
rounded to bf16 before the value product, fp32 sums.
"""

import math

import torch

BF16, F32 = torch.bfloat16, torch.float32
LOG2E = 1.4426950408889634


def cdiv(a, b):
    return -(-a // b)


def default_config(batch, kv_heads, capacity):
    """decode_attention.py:152-157: (block_n, splits, warps)."""
    block_n = 32 if batch * kv_heads < 16 else 64
    splits = min(32, cdiv(256, batch * kv_heads), cdiv(capacity, block_n))
    return block_n, splits, 4


def interval(query, key, value, visible, scale):
    """references.py:195-205: (accumulator [Q,D], maximum [Q], denominator [Q])."""
    count = query.shape[0]
    if key.shape[0] == 0:
        return query.new_zeros((count, query.shape[1]), dtype=F32), torch.full((count,), -math.inf), torch.zeros(count)
    scores = (query.to(F32) @ key.to(F32).T) * (scale * LOG2E)
    scores = torch.where(visible, scores, torch.tensor(-math.inf))
    maximum = scores.max(dim=1).values
    pivot = torch.where(maximum == -math.inf, torch.zeros(()), maximum)
    probabilities = torch.exp2(scores - pivot[:, None])
    return probabilities.to(BF16).to(F32) @ value.to(F32), maximum, probabilities.sum(1)


def merge(partial, stats):
    """references.py:231-238 / decode_attention.py:119-127: [..., S, Q, D], [..., S, Q, 2] -> [..., Q, D]."""
    maxima, denominators = stats[..., 0], stats[..., 1]
    maximum = maxima.max(dim=-2, keepdim=True).values
    correction = torch.exp2(maxima - maximum)
    denominator = (denominators * correction).sum(-2)
    numerator = (partial * correction[..., None]).sum(-3)
    return numerator / denominator[..., None]


def decode_attention(query, key, value, position, scale, splits=None):
    """Q [B,Hq,1,D], KV [B,Hkv,C,D], position int64 [1] or [B] -> bf16 [B,1,Hq,D].

    ``splits`` defaults to the reference's `_default_config`; a per-row ``position`` gives
    row b the valid length position[b] + 1 (the ragged extension of the same rule).
    """
    batch, query_heads, _, dim = query.shape
    kv_heads, capacity = key.shape[1:3]
    groups = query_heads // kv_heads
    if splits is None:
        splits = default_config(batch, kv_heads, capacity)[1]
    chunk = cdiv(capacity, splits)
    pos = position.reshape(-1).to(torch.int64)
    q = query.reshape(batch, kv_heads, groups, dim)
    partial = torch.zeros((batch, kv_heads, splits, groups, dim), dtype=F32)
    stats = torch.zeros((batch, kv_heads, splits, groups, 2), dtype=F32)
    for b in range(batch):
        valid = int(pos[b if pos.numel() > 1 else 0]) + 1
        for s in range(splits):
            begin = s * chunk
            end = max(begin, min(begin + chunk, capacity, valid))
            visible = torch.ones((groups, end - begin), dtype=torch.bool)
            for h in range(kv_heads):
                acc, maximum, denominator = interval(q[b, h], key[b, h, begin:end], value[b, h, begin:end], visible, scale)
                partial[b, h, s], stats[b, h, s, :, 0], stats[b, h, s, :, 1] = acc, maximum, denominator
    out = merge(partial, stats)  # [B, Hkv, G, D]
    return out.reshape(batch, 1, query_heads, dim).to(BF16)


def grouped_sdpa_masked(query, key, value, position, scale):
    """The reference's eager single-token path (engine/attention.py:27-39): each KV group's
    query heads are SDPA rows against the shared K/V head, with a length mask per row."""
    batch, query_heads, _, dim = query.shape
    kv_heads, capacity = key.shape[1:3]
    groups = query_heads // kv_heads
    pos = position.reshape(-1).to(torch.int64)
    lengths = (pos if pos.numel() > 1 else pos.expand(batch)) + 1
    mask = (torch.arange(capacity)[None, :] < lengths[:, None]).view(batch, 1, 1, capacity)
    grouped = query.reshape(batch, kv_heads, groups, dim)
    keys = torch.where(mask.view(batch, 1, capacity, 1), key, torch.zeros((), dtype=key.dtype))
    values = torch.where(mask.view(batch, 1, capacity, 1), value, torch.zeros((), dtype=value.dtype))
    out = torch.nn.functional.scaled_dot_product_attention(
        grouped, keys, values, attn_mask=mask, dropout_p=0.0, is_causal=False, scale=scale
    )
    return out.reshape(batch, 1, query_heads, dim)


def block_attention(query, key, value, position, scale, chain, splits=1):
    """Verify attention: Q token-major [B,T,Hq,D], KV [B,Hkv,C,D], position/chain int64 [B].

    Token t of row b sits at slot position[b] + t. Tokens t < chain[b] see slots
    [0, position[b] + t]; the others see [0, position[b]] plus their own slot
    (decode_attention.py:286-292, :323; references.py:266-285). Returns bf16 [B,T,Hq,D].
    """
    batch, tokens, query_heads, dim = query.shape
    kv_heads, capacity = key.shape[1:3]
    groups = query_heads // kv_heads
    members = tokens * groups
    chunk = cdiv(capacity, splits)
    q = query.reshape(batch, tokens, kv_heads, groups, dim)
    token = torch.arange(members) // groups
    out = torch.zeros((batch, tokens, kv_heads, groups, dim), dtype=F32)
    for row in range(batch):
        first = int(position[row]) + 1
        chained = token < int(chain[row])
        valid = first + torch.where(chained, token, torch.zeros_like(token))
        own = torch.where(chained, torch.full_like(token, -1), first - 1 + token)
        for head in range(kv_heads):
            qm = q[row, :, head].reshape(members, dim)
            partial = torch.zeros((splits, members, dim), dtype=F32)
            stats = torch.zeros((splits, members, 2), dtype=F32)
            for s in range(splits):
                begin = s * chunk
                end = max(begin, min(begin + chunk, capacity, first + tokens - 1))
                slots = torch.arange(begin, end)
                visible = (slots[None, :] < valid[:, None]) | (slots[None, :] == own[:, None])
                acc, maximum, denominator = interval(qm, key[row, head, begin:end], value[row, head, begin:end], visible, scale)
                partial[s], stats[s, :, 0], stats[s, :, 1] = acc, maximum, denominator
            if splits == 1:
                result = partial[0] / stats[0, :, 1][:, None]
            else:
                result = merge(partial, stats)
            out[row, :, head] = result.view(tokens, groups, dim)
    return out.reshape(batch, tokens, query_heads, dim).to(BF16)
