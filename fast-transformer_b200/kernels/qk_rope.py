"""Q/K head RMSNorm, RoPE and in-place KV-cache update on B200.

Drop-in for engine/kernels/qk_rope.py:87-129 (same signature, asserts and return value):
one launch of fb_qk_norm_rope_append writes token-major Q and appends K (normed, rotated)
and V (copied) at each token's cache slot.
"""

import torch

from kernels import _native
from kernels._native import check, lib, ptr, stream
from kernels.merged import Split, source


def qk_rope_cache(packed, q_norm, k_norm, cos, sin, position, keys, values, q_heads, prefill=False, rows=False, phases=None):
    """BF16 packed QKV and [B,Hkv,C,D] caches, for prefill or one decode token.

    Native BF16 phases [1,T,D] are shared by batch rows. Prefill writes [0,T); decode
    writes T slots starting at the device-side scalar position (per row with ``rows``).
    Return a [B,Hq,T,D] view of token-major Q storage (contiguous when T is one).
    """
    batch, kv_heads, capacity, dim = keys.shape
    split = isinstance(packed, Split)
    packed, splits, count, shape = source(packed)
    tokens = shape[1]
    assert keys.dtype == values.dtype == torch.bfloat16
    assert packed.dtype == (torch.float32 if split else torch.bfloat16)
    assert packed.is_contiguous() and keys.is_contiguous() and values.is_contiguous()
    assert shape == (batch, tokens, (q_heads + 2 * kv_heads) * dim)
    assert 0 < tokens <= capacity
    assert values.shape == keys.shape and dim % 2 == 0
    assert not (rows and prefill)
    table = phases is not None
    if table:
        assert rows and phases.shape == (batch, tokens) and phases.is_contiguous() and phases.dtype == torch.int64
        assert cos.shape == sin.shape and cos.shape[-1] == dim and cos.numel() // dim >= capacity
    else:
        assert cos.numel() == sin.numel() == (batch if rows else 1) * tokens * dim
    assert cos.is_contiguous() and sin.is_contiguous()
    assert position.shape == ((tokens,) if prefill else (batch,) if rows else (1,))
    assert position.dtype == torch.int64
    _native.require_cuda(packed, keys, values, cos, sin, position)
    query = torch.empty((batch, tokens, q_heads, dim), device=packed.device, dtype=keys.dtype)
    mode = 1 if prefill else 2 if rows else 0
    check(lib.fb_qk_norm_rope_append(
        ptr(packed), splits if packed.dtype == torch.float32 else 0, ptr(q_norm.weight), ptr(k_norm.weight),
        float(q_norm.variance_epsilon), float(k_norm.variance_epsilon), ptr(cos), ptr(sin),
        ptr(position), ptr(phases) if table else None, ptr(query), ptr(keys), ptr(values),
        batch, tokens, q_heads, kv_heads, dim, capacity, mode, 1 if table else 0, stream(),
    ), "fb_qk_norm_rope_append")
    return query.transpose(1, 2)
