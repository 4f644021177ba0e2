"""fb_prefill_attention (tcgen05 causal GQA flash forward) against a plain PyTorch fp32
reference of the reference's prefill (engine/attention.py:8-21: SDPA, is_causal, GQA):
ragged tile ends, NaN-poisoned cache slots past the prompt, cache views with a larger
capacity, and the config-4 prompt length."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def fp32_causal_gqa(q, k, v, scale):
    batch, q_heads, tokens, dim = q.shape
    groups = q_heads // k.shape[1]
    kk = k[:, :, :tokens].float().repeat_interleave(groups, 1)
    vv = v[:, :, :tokens].float().repeat_interleave(groups, 1)
    s = torch.einsum("bhtd,bhsd->bhts", q.float(), kk) * scale
    mask = torch.ones(tokens, tokens, dtype=torch.bool, device=q.device).triu(1)
    s.masked_fill_(mask, float("-inf"))
    return torch.einsum("bhts,bhsd->bhtd", torch.softmax(s, -1), vv).transpose(1, 2)  # [B, T, Hq, D]


@pytest.mark.parametrize("batch,q_heads,kv_heads,tokens,capacity,dim", [
    (1, 8, 2, 300, 300, 128), (2, 32, 8, 1024, 1100, 128), (1, 4, 4, 127, 200, 128), (3, 16, 2, 129, 129, 128),
    (1, 32, 8, 1, 64, 128), (2, 8, 2, 333, 400, 64), (1, 16, 8, 4096, 4096, 64)])
def test_prefill_attention_matches_fp32_reference(batch, q_heads, kv_heads, tokens, capacity, dim):
    from kernels.prefill import prefill_attention
    g = torch.Generator(device=DEV).manual_seed(tokens + capacity)
    q = torch.randn(batch, q_heads, tokens, dim, device=DEV, generator=g).bfloat16()
    k = torch.randn(batch, kv_heads, capacity, dim, device=DEV, generator=g).bfloat16()
    v = torch.randn(batch, kv_heads, capacity, dim, device=DEV, generator=g).bfloat16()
    k[:, :, tokens:] = float("nan")  # cache slots past the prompt never enter
    v[:, :, tokens:] = float("nan")
    scale = 1 / math.sqrt(dim)
    out = prefill_attention(q, k[:, :, :tokens], v[:, :, :tokens], scale)
    expect = fp32_causal_gqa(q, k, v, scale)
    assert out.shape == (batch, tokens, q_heads, dim)
    assert torch.isfinite(out.float()).all()
    torch.testing.assert_close(out.float(), expect, atol=2e-2, rtol=2e-2)
    from kernels._native import device_error
    assert device_error() == 0


def test_prefill_attention_config4_prompt_against_sdpa():
    """One config-4 row: 8192 tokens, 32/8 heads, against torch SDPA (the reference's own call)."""
    from kernels.prefill import prefill_attention
    g = torch.Generator(device=DEV).manual_seed(8192)
    q = torch.randn(1, 32, 8192, 128, device=DEV, generator=g).bfloat16()
    k = torch.randn(1, 8, 8320, 128, device=DEV, generator=g).bfloat16()
    v = torch.randn(1, 8, 8320, 128, device=DEV, generator=g).bfloat16()
    out = prefill_attention(q, k[:, :, :8192], v[:, :, :8192], 1 / math.sqrt(128))
    ref = torch.nn.functional.scaled_dot_product_attention(q, k[:, :, :8192], v[:, :, :8192], is_causal=True,
                                                           scale=1 / math.sqrt(128), enable_gqa=True)
    torch.testing.assert_close(out.float(), ref.transpose(1, 2).float(), atol=2e-2, rtol=2e-2)
