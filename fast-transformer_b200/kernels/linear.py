"""BF16 skinny projections on B200.

Drop-in for engine/kernels/linear.py:489-523 ``linear(x, weight, split_ok)``: all products
accumulate in FP32 and round once to BF16. Decode-sized inputs (<= MAX_ROWS rows, aligned
K/N) run the TMA + mma.sync kernel fb_linear; with ``split_ok`` a split-K result comes
back as a ``Split`` for a consumer kernel to sum (merged.py). Larger row counts (prefill)
stay on cuBLAS through ``F.linear``, exactly as the reference routes them (linear.py:492).
"""

import torch
from torch.nn import functional as F

from kernels import _native
from kernels._native import check, lib, ptr, stream
from kernels.merged import Split

#: Rows the skinny kernel takes (x is staged as 16/32/64-row slabs).
MAX_ROWS = 64
_SPLITS = {}


def splits_for(rows, n, k, device):
    key = (device, rows, n, k)
    if key not in _SPLITS:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("projection selection must finish during eager warmup")
        _SPLITS[key] = int(lib.fb_linear_splits(rows, n, k))
    return _SPLITS[key]


def supported(rows, weight):
    n, k = weight.shape
    return 0 < rows <= MAX_ROWS and k % 8 == 0 and n % 8 == 0 and weight.dtype == torch.bfloat16


def project(flat, weight, splits, out_fp32=False):
    """fb_linear on [M,K] x [N,K]: BF16 [M,N] (one split) or FP32 partials [S,M,N]."""
    m, k = flat.shape
    n = weight.shape[0]
    if splits == 1 and not out_fp32:
        out = torch.empty((m, n), device=flat.device, dtype=torch.bfloat16)
    else:
        out = torch.empty((splits, m, n), device=flat.device, dtype=torch.float32)
    check(lib.fb_linear(ptr(flat), ptr(weight), ptr(out), m, n, k, splits, 1 if out_fp32 else 0, stream()),
          "fb_linear")
    return out


def merge(partial, out_fp32=False):
    """Sum FP32 partials [S,M,N] in split order into BF16 (or FP32) [M,N]."""
    splits, m, n = partial.shape
    out = torch.empty((m, n), device=partial.device, dtype=torch.float32 if out_fp32 else torch.bfloat16)
    check(lib.fb_merge_splits(ptr(partial), splits, m * n, ptr(out), 1 if out_fp32 else 0, stream()),
          "fb_merge_splits")
    return out


def linear(x, weight, split_ok=False):
    """x @ weight.T in BF16. With ``split_ok`` the result may be a ``Split`` for a consumer kernel."""
    rows = x.numel() // x.shape[-1]
    if x.dtype != torch.bfloat16 or not weight.is_contiguous() or not supported(rows, weight):
        return F.linear(x, weight)
    _native.require_cuda(x, weight)
    flat = x.reshape(rows, x.shape[-1]).contiguous()
    splits = splits_for(rows, weight.shape[0], weight.shape[1], x.device)
    result = project(flat, weight, splits)
    if splits > 1 and split_ok:
        return Split(result, (*x.shape[:-1], weight.shape[0]))
    if splits > 1:
        result = merge(result)
    return result.reshape(*x.shape[:-1], weight.shape[0])
