"""SwiGLU from packed gate/up projections on B200, preserving the SiLU BF16 output.

Drop-in for engine/kernels/swiglu.py:27-40; the kernel is fb_swiglu.
"""

import torch

from kernels import _native
from kernels._native import check, lib, ptr, stream
from kernels.merged import Split, source


def swiglu(packed):
    """Contiguous BF16 [..., 2*I] gate/up input (or its Split partials); new contiguous [..., I] output."""
    split = isinstance(packed, Split)
    packed, splits, count, shape = source(packed)
    width = shape[-1] // 2
    assert packed.is_contiguous() and packed.dtype == (torch.float32 if split else torch.bfloat16)
    _native.require_cuda(packed)
    output = torch.empty((*shape[:-1], width), device=packed.device, dtype=torch.bfloat16)
    rows = output.numel() // width
    check(lib.fb_swiglu(ptr(packed), splits if packed.dtype == torch.float32 else 0, ptr(output), rows, width, stream()), "fb_swiglu")
    return output
