"""Programmatic dependent launch check with the reference's interface (engine/kernels/pdl.py:120-160).

Every libfastb200 kernel is launched with programmatic stream serialization and waits
(``griddepcontrol.wait``) before it touches anything an earlier kernel of the stream writes, so
PDL is always on; there is no per-kernel launcher to patch. ``self_test`` keeps the reference's
contract - called once before the engine builds anything, it checks on a captured two-kernel
chain that dependent kernels still see their producer's results - and uses the library's own
kernels for the chain: fb_merge_splits writes a stage buffer that the next fb_merge_splits
reads. A wrong result raises (these kernels have no non-PDL form to fall back to).
"""

import torch

from kernels import _native
from kernels._native import check, lib, ptr, stream

#: PDL is part of every library kernel's launch.
ENABLED = True


def _chain(value, stage, out, links):
    count = value.numel()
    for _ in range(links):
        check(lib.fb_merge_splits(ptr(value), 1, count, ptr(stage), 1, stream()), "fb_merge_splits")
        check(lib.fb_merge_splits(ptr(stage), 1, count, ptr(out), 1, stream()), "fb_merge_splits")


def self_test(device, count=1024):
    """True once a captured chain of dependent library kernels replays with the expected values
    on ``device`` (20 replays, each after the input changed). False without CUDA; raises
    RuntimeError if a dependent kernel read stale data."""
    if not torch.cuda.is_available():
        return False
    device = torch.device(device)
    value = torch.zeros(count, dtype=torch.float32, device=device)
    stage = torch.zeros_like(value)
    out = torch.zeros_like(value)
    side = torch.cuda.Stream(device=device)
    side.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.device(device), torch.cuda.stream(side):
        _chain(value, stage, out, 3)
        side.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            _chain(value, stage, out, 8)
    expected = torch.arange(count, dtype=torch.float32, device=device)
    for trial in range(20):
        value.copy_(expected + trial)
        graph.replay()
        torch.cuda.synchronize(device)
        if not torch.equal(out, expected + trial):
            raise RuntimeError("programmatic launch let a dependent kernel read stale data")
    del graph
    if _native.device_error() != 0:
        raise RuntimeError("the PDL check raised the library's device error word")
    print("PDL: programmatic dependent launch is on", flush=True)
    return True
