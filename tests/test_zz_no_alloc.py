"""The no-allocation decode attention entry point (fb_decode_attention_noalloc), called
through the C ABI. It exists for callers that cannot allocate device memory on their call
path: hosts that own a fixed device pool and hand the library only inputs and outputs, or
plugin hosts whose allocator the plugin may not call. Its scratch is a fixed array inside
libfastb200.so, so its output must equal the allocating entry point's (fb_decode_attention,
which takes a caller-provided workspace) on consecutive calls that share that array.

Collected last on purpose (file name), so a stop-at-first-failure run has run everything else.
"""

import ctypes
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _inputs(lengths, q_heads, kv_heads, dim, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    batch, capacity = len(lengths), max(lengths)
    q = torch.randn(batch, q_heads, 1, dim, device="cuda", generator=g).to(torch.bfloat16)
    k = torch.randn(batch, kv_heads, capacity, dim, device="cuda", generator=g).to(torch.bfloat16)
    v = torch.randn(batch, kv_heads, capacity, dim, device="cuda", generator=g).to(torch.bfloat16)
    for b, n in enumerate(lengths):  # unused slots must never be read
        k[b, :, n:] = float("nan")
        v[b, :, n:] = float("nan")
    position = torch.tensor([n - 1 for n in lengths], dtype=torch.int64, device="cuda")
    return q, k, v, position


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")
def test_no_alloc_entry_point_matches_allocating_entry_point_on_consecutive_calls():
    from kernels import _native
    from kernels.decode_attention import attend

    fn = _native.lib.fb_decode_attention_noalloc
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    # Two calls in a row with different shapes: the second finds the first one's leftovers
    # in the shared scratch array.
    for lengths, q_heads, kv_heads, dim, seed in (([5000, 1, 700, 64], 32, 8, 128, 1), ([8192, 65], 16, 8, 64, 2)):
        q, k, v, position = _inputs(lengths, q_heads, kv_heads, dim, seed)
        batch, capacity, scale = len(lengths), k.shape[2], 1.0 / math.sqrt(dim)
        out = torch.full((batch, 1, q_heads, dim), float("nan"), dtype=torch.bfloat16, device="cuda")
        status = fn(q.data_ptr(), k.data_ptr(), v.data_ptr(), position.data_ptr(), 1, out.data_ptr(), batch,
                    q_heads, kv_heads, dim, capacity, scale, stream)
        assert status == 0, _native._STATUS.get(status, status)
        expected = attend(q, k, v, position, scale)  # fb_decode_attention with its own workspace
        torch.cuda.synchronize()
        assert torch.isfinite(out.float()).all()
        torch.testing.assert_close(out.float(), expected.float(), atol=2e-2, rtol=2e-2)
    assert _native.device_error() == 0

    # Beyond the fixed limit (batch * kv_heads > 512): a clear error and nothing launched.
    big = fn(q.data_ptr(), k.data_ptr(), v.data_ptr(), position.data_ptr(), 0, out.data_ptr(), 65, 64, 8, 128,
             16, 0.1, stream)
    assert big == -6
