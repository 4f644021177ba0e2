"""Split-KV GQA decode attention on B200: drop-in for engine/kernels/decode_attention.py.

``decode_attention`` keeps the reference signature and contract
(engine/kernels/decode_attention.py:238-257): BF16 Q [B,Hq,1,D], a contiguous BF16 layer
cache [B,Hkv,C,D] and a device-side int64 ``position``; every valid slot [0, position]
contributes; the result is a new [B,1,Hq,D] tensor. Additionally ``position`` may hold
one entry per row ([B]) for ragged batches. The kernels are fb_decode_attention (TMA +
mma.sync partials over a balanced persistent split) and fb_decode_attention_combine
(log-sum-exp merge), launched on the current stream, so CUDA-graph capture records them.
"""

import torch

from kernels import _native
from kernels._native import check, lib, ptr, stream

_CTAS = {}


def _ctas(shape):
    """Persistent CTA count per (device, B, Hkv, C, D): fixed before capture, like the
    reference's per-shape layout choice (decode_attention.py:247-256)."""
    if shape not in _CTAS:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("attention layout selection must finish during eager warmup")
        _, batch, kv_heads, capacity, dim = shape
        _CTAS[shape] = int(lib.fb_decode_attention_ctas(batch, kv_heads, capacity, dim))
    return _CTAS[shape]


def workspace_bytes(batch, query_heads, kv_heads, dim, ctas):
    return int(lib.fb_decode_attention_workspace(batch, query_heads, kv_heads, dim, ctas))


def attend(query, key, value, position, scale, out=None, workspace=None, ctas=None, two_launch=False):
    """Launch decode attention. ``query`` [B,Hq,1,D] or [B,Hq,D]; returns ``out`` [B,1,Hq,D].

    One launch by default (fb_decode_attention, merge fused into the last CTA of each pair);
    ``two_launch`` runs fb_decode_attention_partials then fb_decode_attention_combine. A
    caller-provided ``workspace`` must have been zeroed before its first fused use.
    """
    batch, query_heads, dim = query.shape[0], query.shape[1], query.shape[-1]
    kv_heads, capacity = key.shape[1], key.shape[2]
    if ctas is None:
        ctas = _ctas((query.device, batch, kv_heads, capacity, dim))
    need = workspace_bytes(batch, query_heads, kv_heads, dim, ctas)
    if workspace is None:
        workspace = torch.zeros(need, dtype=torch.uint8, device=query.device)
    if out is None:
        out = torch.empty((batch, 1, query_heads, dim), device=query.device, dtype=query.dtype)
    per_row = 1 if position.numel() > 1 else 0
    s = stream()
    args = (ptr(query), ptr(key), ptr(value), ptr(position), per_row, ptr(out), ptr(workspace), workspace.numel(),
            batch, query_heads, kv_heads, dim, capacity, float(scale), ctas, s)
    if not two_launch:
        check(lib.fb_decode_attention(*args), "fb_decode_attention")
        return out
    check(lib.fb_decode_attention_partials(*args), "fb_decode_attention_partials")
    check(lib.fb_decode_attention_combine(ptr(position), per_row, ptr(out), ptr(workspace), workspace.numel(),
                                          batch, query_heads, kv_heads, dim, capacity, ctas, s),
          "fb_decode_attention_combine")
    return out


def decode_attention(query, key, value, position, scale):
    """Q [B,Hq,1,D], KV [B,Hkv,C,D] -> [B,1,Hq,D]."""
    batch, query_heads, tokens, dim = query.shape
    kv_heads, capacity = key.shape[1:3]
    assert tokens == 1 and query_heads % kv_heads == 0
    assert query.dtype == key.dtype == value.dtype == torch.bfloat16
    assert query.is_contiguous() and key.is_contiguous() and value.is_contiguous()
    assert value.shape == key.shape and key.shape[0] == batch and key.shape[3] == dim
    assert dim in (64, 128) and position.dtype == torch.int64
    assert position.shape == (1,) or position.shape == (batch,)
    assert position.is_contiguous()
    _native.require_cuda(query, key, value, position)
    return attend(query, key, value, position, scale)


_BLOCK_SPLITS = {}


def block_attention(query, key, value, position, scale, chain, splits=None):
    """Verify blocks: token-major Q [B,T,Hq,D], KV [B,Hkv,C,D], position [B] -> [B,T,Hq,D].

    Token t of row b occupies slot ``position[b] + t``. The first ``chain[b]`` tokens attend
    causally; the rest are alternatives to token 1 and attend to the prefix through token 0
    plus themselves. The block's own keys must already be in the cache. The kernel is
    fb_verify_attention (tcgen05 UMMA, TMEM accumulators), plus its split merge.
    """
    batch, tokens, query_heads, dim = query.shape
    kv_heads, capacity = key.shape[1:3]
    assert key.shape[0] == batch and query_heads % kv_heads == 0
    assert query.dtype == key.dtype == value.dtype == torch.bfloat16
    assert query.is_contiguous() and key.is_contiguous() and value.is_contiguous()
    assert value.shape == key.shape and key.shape[3] == dim and dim in (64, 128)
    assert position.shape == (batch,) and position.dtype == torch.int64
    assert chain.shape == (batch,) and chain.dtype == torch.int64
    _native.require_cuda(query, key, value, position, chain)
    shape = (query.device, batch, tokens, query_heads, kv_heads, capacity, dim)
    if splits is None:
        if shape not in _BLOCK_SPLITS:
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError("attention layout selection must finish during eager warmup")
            _BLOCK_SPLITS[shape] = int(lib.fb_verify_attention_splits(batch, tokens, kv_heads, capacity))
        splits = _BLOCK_SPLITS[shape]
    out = torch.empty((batch, tokens, query_heads, dim), device=query.device, dtype=query.dtype)
    need = int(lib.fb_verify_attention_workspace(batch, tokens, query_heads, kv_heads, splits))
    workspace = torch.empty(need if splits > 1 else 0, dtype=torch.uint8, device=query.device)
    check(lib.fb_verify_attention(ptr(query), ptr(key), ptr(value), ptr(position), ptr(chain), ptr(out),
                                  ptr(workspace) if splits > 1 else None, workspace.numel(), batch, tokens,
                                  query_heads, kv_heads, dim, capacity, float(scale), splits, stream()),
          "fb_verify_attention")
    if splits > 1:
        _native.launches += 1  # the split merge
    return out
