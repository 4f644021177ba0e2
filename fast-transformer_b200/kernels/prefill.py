"""Causal GQA prefill attention on B200 (fb_prefill_attention, tcgen05 flash forward).

Replaces the prefill call of engine/attention.py:8-21 (`grouped_sdpa` without a mask, i.e.
torch SDPA's Flash backend with is_causal and enable_gqa) for head_dim 64 and 128.
"""

import torch

from kernels import _native
from kernels._native import check, lib, ptr, stream


def prefill_attention(query, key, value, scale):
    """query [B, Hq, T, D], key/value [B, Hkv, C, D] with the prompt in slots [0, T) (C >= T;
    a slice key[:, :, :T] of a larger cache is accepted) -> [B, T, Hq, D] bf16, causal."""
    batch, q_heads, tokens, dim = query.shape
    kv_heads = key.shape[1]
    assert query.dtype == key.dtype == value.dtype == torch.bfloat16
    assert key.shape[0] == batch and value.shape == key.shape and q_heads % kv_heads == 0 and dim in (64, 128)
    _native.require_cuda(query, key, value)
    # The kernel reads K/V through the cache's own row pitch: a [:, :, :T] view of a contiguous
    # [B, Hkv, C, D] store is used in place (C = its capacity); anything else is copied.
    capacity = key.stride(1) // dim if key.stride(1) % dim == 0 else None
    contiguous_rows = (key.stride(-1) == 1 and key.stride(2) == dim and capacity is not None and capacity >= tokens
                       and key.stride(0) == kv_heads * key.stride(1) and value.stride() == key.stride())
    if not contiguous_rows:
        key, value = key.contiguous(), value.contiguous()
        capacity = key.shape[2]
    q = query.contiguous()
    out = torch.empty((batch, tokens, q_heads, dim), dtype=torch.bfloat16, device=query.device)
    check(lib.fb_prefill_attention(ptr(q), ptr(key), ptr(value), ptr(out), batch, tokens, q_heads, kv_heads, dim,
                                   capacity, float(scale), stream()), "fb_prefill_attention")
    return out
