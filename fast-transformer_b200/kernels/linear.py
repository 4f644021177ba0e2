"""BF16 skinny projections on B200.

Drop-in for engine/kernels/linear.py:489-523 ``linear(x, weight, split_ok)``: all products
accumulate in FP32 and round once to BF16. Decode-sized inputs (<= MAX_ROWS rows, aligned
K/N) run the TMA + mma.sync kernel fb_linear over (N/128 tiles) x (K splits); with
``split_ok`` a split-K result comes back as a ``Split`` of FP32 partials for a consumer kernel
to sum (merged.py), otherwise the split CTAs of each tile form a thread-block cluster that sums
the tile's partials in split order and writes BF16 (same launch). Larger row counts (prefill)
stay on cuBLAS through ``F.linear``, exactly as the reference routes them (linear.py:492).

``keep_native`` is the reference's hook for leaving a shape on cuBLAS without tuning it
(linear.py:484-486); the B200 kernels choose their launch shape by a fixed rule (no timed
search), so it only records the request.
"""

import torch
from torch.nn import functional as F

from kernels import _native
from kernels._native import check, lib, ptr, stream
from kernels.merged import Split

#: Rows the skinny kernel takes (x is staged as 16/32/64-row slabs).
MAX_ROWS = 64
BF16_OUT, FP32_OUT, SWIGLU_OUT, SPLITS_OUT = 0, 1, 2, 3
_SPLITS = {}


def splits_for(rows, n, k, device, finished=False):
    """fb_linear_splits' choice, or fb_linear_finished_splits' for finished-tile epilogues."""
    key = (device, rows, n, k, finished)
    if key not in _SPLITS:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("projection selection must finish during eager warmup")
        choose = lib.fb_linear_finished_splits if finished else lib.fb_linear_splits
        _SPLITS[key] = int(choose(rows, n, k))
    return _SPLITS[key]


def keep_native(rows, weight):
    """engine/kernels/linear.py:484-486: leave ``rows`` x ``weight`` on cuBLAS without spending
    tuning time on it. The B200 projection has no timed search to skip, and the reference calls
    this only for row counts above MAX_ROWS (its verify blocks), which ``linear`` already routes
    to cuBLAS; the shape is recorded so ``linear`` keeps it there whatever its row count."""
    _NATIVE.add((weight.device, rows, weight.shape[0], weight.shape[1]))


_NATIVE = set()


def supported(rows, weight):
    n, k = weight.shape
    return 0 < rows <= MAX_ROWS and k % 8 == 0 and n % 8 == 0 and weight.dtype == torch.bfloat16


def project(flat, weight, epilogue=BF16_OUT, splits=None):
    """fb_linear on [M,K] x [N,K]: BF16 [M,N], FP32 [M,N], SwiGLU BF16 [M,N/2] or FP32 split
    partials [S,M,N]."""
    m, k = flat.shape
    n = weight.shape[0]
    if splits is None:
        splits = splits_for(m, n, k, flat.device, finished=epilogue != SPLITS_OUT)
    if epilogue == SWIGLU_OUT:
        out = torch.empty((m, n // 2), device=flat.device, dtype=torch.bfloat16)
    elif epilogue == SPLITS_OUT:
        out = torch.empty((splits, m, n), device=flat.device, dtype=torch.float32)
    else:
        out = torch.empty((m, n), device=flat.device, dtype=torch.float32 if epilogue == FP32_OUT else torch.bfloat16)
    check(lib.fb_linear(ptr(flat), ptr(weight), ptr(out), m, n, k, epilogue, splits, stream()), "fb_linear")
    return out


def linear(x, weight, split_ok=False):
    """x @ weight.T in BF16. With ``split_ok`` the result may be a ``Split`` for a consumer kernel."""
    rows = x.numel() // x.shape[-1]
    if x.dtype != torch.bfloat16 or not weight.is_contiguous() or not supported(rows, weight):
        return F.linear(x, weight)
    if _NATIVE and (weight.device, rows, weight.shape[0], weight.shape[1]) in _NATIVE:
        return F.linear(x, weight)
    _native.require_cuda(x, weight)
    flat = x.reshape(rows, x.shape[-1]).contiguous()
    n, k = weight.shape
    splits = splits_for(rows, n, k, x.device)
    if split_ok and splits > 1:
        return Split(project(flat, weight, SPLITS_OUT, splits), (*x.shape[:-1], n))
    return project(flat, weight, BF16_OUT, splits_for(rows, n, k, x.device, finished=True)).reshape(
        *x.shape[:-1], n)


def swiglu_linear(x, gate_up_blocked):
    """SwiGLU(x @ W^T), W's rows being [gate; up] interleaved in 64-row blocks: bf16(bf16(silu(
    gate)) * up) per feature, the reference's projection + swiglu arithmetic. At one K split the
    projection's epilogue applies SwiGLU (one launch). With K splits the projection writes
    split partials that fb_swiglu_blocked sums and activates (measured faster inside the decode
    step than summing the splits in the projection's own launch). The same bits either way."""
    rows = x.numel() // x.shape[-1]
    flat = x.reshape(rows, x.shape[-1]).contiguous()
    n, k = gate_up_blocked.shape
    splits = splits_for(rows, n, k, x.device)
    if splits == 1:
        return project(flat, gate_up_blocked, SWIGLU_OUT, splits).reshape(*x.shape[:-1], n // 2)
    partials = project(flat, gate_up_blocked, SPLITS_OUT, splits)
    out = torch.empty((rows, n // 2), device=x.device, dtype=torch.bfloat16)
    check(lib.fb_swiglu_blocked(ptr(partials), splits, ptr(out), rows, n // 2, stream()), "fb_swiglu_blocked")
    return out.reshape(*x.shape[:-1], n // 2)
