"""tcgen05 verify (q_len > 1) attention against the reference's block attention (golden
fixtures made by running the reference's code) and the CPU oracle: BASELINE config 5 plus
the reference's mask cases (chain = T, T-2, 2, 1; position 0; several splits; 1e6 tails)."""

import math
import os

import pytest
import torch

import cases
from oracle import attention as oatt

pytestmark = pytest.mark.gpu
GOLDEN = os.path.dirname(os.path.abspath(cases.__file__))
TOL = dict(atol=2e-2, rtol=2e-2)


@pytest.fixture(autouse=True)
def _no_device_errors():
    from kernels import _native
    _native.device_error()
    yield
    assert _native.device_error() == 0, "a kernel raised its device error word"


@pytest.mark.parametrize("case", cases.BLOCK_CASES, ids=[c[0] for c in cases.BLOCK_CASES])
def test_verify_attention_matches_reference(case):
    from kernels.decode_attention import block_attention
    fx = torch.load(os.path.join(GOLDEN, "block.pt"), weights_only=False)[case[0]]
    q, k, v, position, chain, scale, splits = cases.block_inputs(case)
    assert cases.digest(q, k, v, position, chain) == fx["digest"]
    args = (q.cuda(), k.cuda(), v.cuda(), position.cuda(), scale, chain.cuda())
    outs = [block_attention(*args)]                       # default split count
    for s in sorted({1, splits, 3}):
        outs.append(block_attention(*args, splits=s))
    for out in outs:
        out = out.cpu()
        assert torch.isfinite(out.float()).all()
        torch.testing.assert_close(out.float(), fx["out"].float(), **TOL)


@pytest.mark.parametrize("d", [128, 64])
def test_verify_attention_two_member_groups_and_graph(d):
    """T*G = 64 members (two 32-member CTA groups), ragged positions, captured in a graph."""
    from kernels.decode_attention import block_attention
    g = torch.Generator().manual_seed(9)
    batch, tokens, hq, hkv, cap = 3, 16, 32, 8, 700
    q = torch.randn(batch, tokens, hq, d, generator=g).bfloat16()
    k = torch.randn(batch, hkv, cap, d, generator=g).bfloat16()
    v = torch.randn(batch, hkv, cap, d, generator=g).bfloat16()
    position = torch.tensor([600, 0, 333])
    chain = torch.tensor([16, 5, 1])
    expect = oatt.block_attention(q, k, v, position, 1 / math.sqrt(d), chain)
    args = (q.cuda(), k.cuda(), v.cuda(), position.cuda(), 1 / math.sqrt(d), chain.cuda())
    eager = block_attention(*args)
    torch.testing.assert_close(eager.cpu().float(), expect.float(), **TOL)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        captured = block_attention(*args)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(captured, eager)



def test_verify_attention_many_splits_deterministic():
    """Five KV splits and two 32-member groups: identical bits on repeated calls and the
    oracle's result (the split merge runs in split order)."""
    from kernels.decode_attention import block_attention
    g = torch.Generator().manual_seed(11)
    batch, tokens, hq, hkv, cap, d = 2, 12, 32, 8, 1500, 128  # 48 members: two groups
    q = torch.randn(batch, tokens, hq, d, generator=g).bfloat16()
    k = torch.randn(batch, hkv, cap, d, generator=g).bfloat16()
    v = torch.randn(batch, hkv, cap, d, generator=g).bfloat16()
    position = torch.tensor([1400, 900])
    chain = torch.tensor([12, 3])
    expect = oatt.block_attention(q, k, v, position, 1 / math.sqrt(d), chain)
    args = (q.cuda(), k.cuda(), v.cuda(), position.cuda(), 1 / math.sqrt(d), chain.cuda())
    first = block_attention(*args, splits=5)
    again = block_attention(*args, splits=5)
    assert torch.equal(first, again)
    torch.testing.assert_close(first.cpu().float(), expect.float(), **TOL)
