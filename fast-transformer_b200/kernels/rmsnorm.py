"""Qwen3's RMSNorm on B200, preserving the reference's BF16 cast boundaries.

Drop-in for engine/kernels/rmsnorm.py (`rms_norm` :49-72, `add_rms_norm` :98-125,
`embed_rms_norm` :145-162): same signatures, same returned tensors, same errors for rows
that do not fit. The kernels are fb_rmsnorm / fb_add_rmsnorm / fb_embed_rmsnorm.
"""

import torch

from kernels import _native
from kernels._native import check, lib, ptr, stream
from kernels.merged import Split, source

#: Widest row the kernels take (8 bf16 per thread chunk, 8 chunks x 256 threads).
MAX_WIDTH = 16384


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """RMSNorm over the last dimension, matching ``Qwen3RMSNorm.forward``."""
    shape = x.shape
    rows = x.reshape(-1, shape[-1]).contiguous()
    n_rows, n_cols = rows.shape
    if n_cols > MAX_WIDTH or n_cols % 8:
        raise ValueError(f"a row must fit in one block; {n_cols} columns does not")
    _native.require_cuda(rows, weight)
    out = torch.empty_like(rows)
    check(lib.fb_rmsnorm(ptr(rows), rows.stride(0), ptr(weight), ptr(out), n_rows, n_cols, float(eps), stream()),
          "fb_rmsnorm")
    return out.reshape(shape)


def add_rms_norm(x, residual, weight, eps):
    """Return (normalized sum, BF16 sum), without mutating either input."""
    x_data, splits, count, shape = source(x)
    assert shape == tuple(residual.shape)
    assert residual.dtype == weight.dtype == torch.bfloat16
    assert x_data.dtype == (torch.float32 if isinstance(x, Split) else torch.bfloat16)
    width = shape[-1]
    if width > MAX_WIDTH or width % 8:
        raise ValueError(f"a row must fit in one block; {width} columns does not")
    x_rows = x_data if isinstance(x, Split) else x_data.reshape(-1, width).contiguous()
    residual_rows = residual.reshape(-1, width).contiguous()
    _native.require_cuda(x_rows, residual_rows, weight)
    out = torch.empty_like(residual_rows)
    summed = torch.empty_like(residual_rows)
    rows = residual_rows.shape[0]
    check(lib.fb_add_rmsnorm(ptr(x_rows), splits if x_data.dtype == torch.float32 else 0, ptr(residual_rows), ptr(weight), ptr(out), ptr(summed),
                             rows, width, float(eps), stream()), "fb_add_rmsnorm")
    return out.reshape(shape), summed.reshape(shape)


def embed_rms_norm(token_ids, table, weight, eps):
    """(normalized, hidden) for the embedding rows of ``token_ids``: one launch instead of a gather and a norm."""
    ids = token_ids.reshape(-1).contiguous()
    n_cols = table.shape[1]
    if n_cols > MAX_WIDTH or n_cols % 8 or not table.is_contiguous() or ids.dtype != torch.int64:
        raise ValueError("embedding rows must fit one block and the table must be contiguous")
    _native.require_cuda(ids, table, weight)
    hidden = torch.empty((ids.numel(), n_cols), dtype=table.dtype, device=table.device)
    out = torch.empty_like(hidden)
    check(lib.fb_embed_rmsnorm(ptr(ids), ptr(table), table.shape[0], ptr(weight), ptr(out), ptr(hidden),
                               ids.numel(), n_cols, float(eps), stream()), "fb_embed_rmsnorm")
    shape = (*token_ids.shape, n_cols)
    return out.reshape(shape), hidden.reshape(shape)
