"""Greedy token ids on B200: torch.argmax's answer over BF16 logits.

Drop-in for engine/kernels/argmax.py:51-70 (`argmax`), :112-129 (`fused_argmax`) and
:132-167 (`greedy_tokens`). Ties resolve to the lowest index at every stage (torch.argmax's
rule); bf16 -> fp32 is exact, so the result equals torch.argmax on the same logits.
``fused_argmax`` never writes the logits: the projection's epilogue reduces each 128-column
tile of bf16-rounded logits (one K split, the projection's own arithmetic at S = 1) to a
per-row candidate, and fb_argmax_candidates picks each row's first best; in tensor
parallelism it also exchanges the ranks' bests over NVLink (vocabulary-parallel LM head).
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


def fused_supported(rows, weight):
    n, k = weight.shape
    return 0 < rows <= 64 and n % 8 == 0 and k % 8 == 0 and weight.dtype == torch.bfloat16 and weight.is_contiguous()


def fused_argmax(x, weight, out=None, index_base=0, exchange=None):
    """argmax(x @ weight.T) per row without materializing the logits; None if not applicable.

    ``out``: int64 [rows] to write (allocated if None). ``index_base``: vocabulary index of
    weight row 0 (a rank's slice). ``exchange``: (world, rank, peer_ptrs, local_ptr, epoch)
    to reduce the ranks' bests over NVLink (every rank then writes the same ids).
    """
    rows, k = x.numel() // x.shape[-1], x.shape[-1]
    if x.dtype != torch.bfloat16 or not fused_supported(rows, weight):
        return None
    _native.require_cuda(x, weight)
    flat = x.reshape(rows, k).contiguous()
    n = weight.shape[0]
    tiles = (n + 127) // 128
    cand = torch.empty(int(lib.fb_argmax_candidates_bytes(rows, n)) // 8, dtype=torch.int64, device=x.device)
    if out is None:
        out = torch.empty(x.shape[:-1], dtype=torch.int64, device=x.device)
    check(lib.fb_linear_argmax(ptr(flat), ptr(weight), rows, n, k, int(index_base), ptr(cand), stream()),
          "fb_linear_argmax")
    if exchange is None:
        check(lib.fb_argmax_candidates(ptr(cand), rows, tiles, 1, 0, None, None, None, ptr(out), None, stream()),
              "fb_argmax_candidates")
    else:
        world, rank, peers, local, epoch = exchange
        check(lib.fb_argmax_candidates(ptr(cand), rows, tiles, world, rank, peers, local, ptr(epoch), ptr(out), None,
                                       stream()), "fb_argmax_candidates")
    return out


def greedy_tokens(x, weight, linear, top=None):
    """Greedy token per row of x @ weight.T.

    With ``top`` the caller also wants each row's winning logit and the logits themselves, so
    the projection path is taken and ``(ids, logits)`` returned, as in the reference.
    Otherwise the fused kernel runs where it applies (its tile arithmetic is the projection's
    at one K split, so no agreement probe is needed), else project + argmax.
    """
    if top is not None:
        logits = linear(x, weight)
        return argmax(logits, top=top), logits
    fused = fused_argmax(x, weight)
    if fused is not None:
        return fused
    return argmax(linear(x, weight))
