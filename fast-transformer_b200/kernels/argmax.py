"""Greedy token ids straight from BF16 logits on B200: torch.argmax's answer in two launches.

Drop-in for engine/kernels/argmax.py:51-70 (`argmax`) and :132-167 (`greedy_tokens`).
Ties resolve to the lowest index at both stages (torch.argmax's rule); bf16 -> fp32 is
exact, so the result equals torch.argmax on the same logits.
"""

import torch

from kernels import _native
from kernels._native import check, lib, ptr, stream


def argmax(logits, block=8192, top=None):
    """int64 argmax over the last dimension of BF16 logits [..., V].

    With ``top``, also writes each row's winning logit there as FP32. ``block`` is kept for
    signature compatibility; the kernel's stage-one block is fixed at 8192 columns.
    """
    if logits.dtype != torch.bfloat16:
        return logits.argmax(dim=-1)
    logits = logits.contiguous()
    _native.require_cuda(logits)
    vocab = logits.shape[-1]
    rows = logits.numel() // vocab
    need = int(lib.fb_argmax_workspace(rows, vocab))
    workspace = torch.empty(need, dtype=torch.uint8, device=logits.device)
    out = torch.empty(logits.shape[:-1], dtype=torch.int64, device=logits.device)
    if top is not None:
        assert top.dtype == torch.float32 and top.numel() >= rows and top.is_contiguous()
    check(lib.fb_argmax(ptr(logits), rows, vocab, ptr(out), ptr(top) if top is not None else None,
                        ptr(workspace), need, stream()), "fb_argmax")
    return out


def greedy_tokens(x, weight, linear, top=None):
    """Greedy token per row of x @ weight.T: project, then argmax.

    With ``top`` the caller also wants each row's winning logit and the logits
    themselves, so ``(ids, logits)`` is returned, as in the reference.
    """
    logits = linear(x, weight)
    if top is not None:
        return argmax(logits, top=top), logits
    return argmax(logits)
