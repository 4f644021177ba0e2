"""Speculation bookkeeping on B200: one launch to propose, one to settle.

Drop-in for engine/kernels/spec.py: ``propose`` (:106-124), ``within_margin`` (:154-166),
``settle`` (:227-240) and ``relocate`` (:262-270), with the same signatures, asserts and
in-place effects, each one fb_spec_* launch of libfastb200 on the current stream.
"""

import torch

from kernels import _native
from kernels._native import check, lib, ptr, stream


def propose(history, position, tokens_per_row, drafts_by_match, successor, stale, chains, phases):
    """Per row: trusted token, chain drafts, alternatives (int64 [B, T]); fills ``chains`` and ``phases``."""
    batch, size = history.shape
    assert history.is_contiguous() and history.dtype == position.dtype == successor.dtype == torch.int64
    assert position.shape == (batch,) and successor.dim() == 2 and successor.is_contiguous()
    assert chains.shape == (batch,) and phases.shape == (batch, tokens_per_row) and phases.is_contiguous()
    assert stale.shape == (batch,) and stale.dtype == torch.int64
    assert len(drafts_by_match) == 4 and all(1 <= d <= tokens_per_row - 1 for d in drafts_by_match)
    _native.require_cuda(history, position, successor, stale, chains, phases)
    tokens = torch.empty((batch, tokens_per_row), dtype=torch.int64, device=history.device)
    d0, d1, d2, d3 = (int(d) for d in drafts_by_match)
    check(lib.fb_spec_propose(ptr(history), size, ptr(position), ptr(successor), successor.shape[0], successor.shape[1],
                              ptr(stale), ptr(tokens), ptr(chains), ptr(phases), batch, tokens_per_row, d0, d1, d2, d3,
                              8, stream()), "fb_spec_propose")
    return tokens


def within_margin(logits, tokens, top, margin):
    """int64 [batch, TOKENS] flags: is chain draft ``slot`` a legal emission? (slot 0: 0)"""
    batch, count = tokens.shape
    vocab = logits.shape[-1]
    assert logits.is_contiguous() and tokens.is_contiguous() and top.is_contiguous()
    assert logits.numel() // vocab == batch * count and top.numel() == batch * count
    assert logits.dtype == torch.bfloat16 and top.dtype == torch.float32
    _native.require_cuda(logits, tokens, top)
    within = torch.empty_like(tokens)
    check(lib.fb_spec_within_margin(ptr(logits), vocab, ptr(tokens), ptr(top), ptr(within), batch, count,
                                    float(margin), stream()), "fb_spec_within_margin")
    return within


def settle(tokens, greedy, position, limit, history, result, move_from, move_to, chains, stale, within=None):
    """Accept, clamp at ``limit``, record emitted tokens, plan the KV move, advance; in place."""
    batch, count = tokens.shape
    assert tokens.is_contiguous() and greedy.is_contiguous() and history.is_contiguous() and result.is_contiguous()
    assert greedy.shape == tokens.shape and result.shape == (batch, count + 1) and chains.shape == (batch,)
    assert tokens.dtype == greedy.dtype == position.dtype == limit.dtype == history.dtype == result.dtype == torch.int64
    assert move_from.dtype == move_to.dtype == torch.int64 and move_from.shape == move_to.shape == (batch,)
    assert stale.shape == (batch,) and stale.dtype == torch.int64
    _native.require_cuda(tokens, greedy, position, limit, history, result, move_from, move_to, chains, stale)
    check(lib.fb_spec_settle(ptr(tokens), ptr(greedy), ptr(within) if within is not None else None, ptr(position),
                             ptr(limit), ptr(history), history.shape[1], ptr(result), ptr(move_from), ptr(move_to),
                             ptr(chains), ptr(stale), batch, count, stream()), "fb_spec_settle")


def relocate(store, move_from, move_to):
    """Copy one K/V slot per row, in every layer: store is [2, L, B, Hkv, C, D]."""
    planes, layers, batch, kv_heads, capacity, dim = store.shape
    assert store.is_contiguous() and planes == 2 and move_from.shape == move_to.shape == (batch,)
    _native.require_cuda(store, move_from, move_to)
    check(lib.fb_spec_relocate(ptr(store), planes * layers, batch, kv_heads, capacity, dim, ptr(move_from),
                               ptr(move_to), stream()), "fb_spec_relocate")
