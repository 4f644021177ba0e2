"""Whole-model GPU parity: the CUDA-graph Qwen3 decode step against the reference's greedy
tokens/logits (tiny model fixtures) and against the CPU oracle (Qwen3-0.6B architecture)."""

import os

import pytest
import torch

import cases
import decode as fdecode
import qwen3
from oracle import model as omodel

pytestmark = pytest.mark.gpu
GOLDEN = os.path.dirname(os.path.abspath(cases.__file__))


def assert_logits_close(actual, expected, chosen, gap=0.02):
    """bf16 logits: error normalised by the logit scale within 2e-2, and the chosen token's
    teacher-forced gap to the row maximum within ``gap`` (agent/verify_gpu.py:221-231 uses 0.02)."""
    scale = expected.abs().max()
    err = (actual - expected).abs().max()
    assert err <= 2e-2 * scale, (err, scale)
    selected = expected.gather(-1, chosen[..., None])[..., 0]
    assert (expected.max(-1).values - selected).max() <= gap


def tiny_state(batch, prompt, steps):
    cfg = qwen3.Config.make(**cases.TINY_QWEN3)
    weights = qwen3.from_state_dict(cfg, cases.tiny_qwen3_weights(), "cuda")
    return fdecode.DecodeState(weights, batch, prompt, steps)


@pytest.mark.parametrize("case", cases.MODEL_CASES, ids=[c[0] for c in cases.MODEL_CASES])
def test_tiny_qwen3_greedy_matches_reference(case):
    fx = torch.load(os.path.join(GOLDEN, "model.pt"), weights_only=False)[case[0]]
    prompt, steps = cases.model_prompt(case)
    state = tiny_state(prompt.shape[0], prompt.shape[1], steps)
    tokens, logits = fdecode.greedy(state, prompt.cuda(), steps)
    tokens, logits = tokens.cpu(), logits.cpu()
    assert torch.equal(tokens, fx["native_tokens"]), (tokens, fx["native_tokens"])
    assert torch.equal(tokens, fx["engine_tokens"])
    assert_logits_close(logits, fx["native_logits"], tokens)


def test_tiny_qwen3_graph_replay_matches_eager_and_host_api():
    prompt, steps = cases.model_prompt(cases.MODEL_CASES[1])
    batch, length = prompt.shape
    eager = tiny_state(batch, length, steps + 4)
    tokens, _ = fdecode.greedy(eager, prompt.cuda(), steps)
    state = tiny_state(batch, length, steps + 4)
    state.prefill(prompt.cuda())
    first = state.token_ids[:, 0].clone()
    state.capture()
    got = [first]
    for _ in range(steps - 1):
        state.step()
        got.append(state.token_ids[:, 0].clone())
    torch.cuda.synchronize()
    assert torch.equal(torch.stack(got, 1).cpu(), tokens.cpu())
    # the host-facing call: pinned ids in, replay, pinned ids out
    state2 = tiny_state(batch, length, steps + 4)
    state2.prefill(prompt.cuda())
    state2.capture()
    host_in = torch.empty(batch, dtype=torch.int64, pin_memory=True)
    host_out = torch.empty(batch, dtype=torch.int64, pin_memory=True)
    host_in.copy_(state2.token_ids[:, 0].cpu())
    seen = [host_in.clone()]
    for _ in range(steps - 1):
        state2.step_host(host_in, host_out)
        torch.cuda.current_stream().synchronize()
        seen.append(host_out.clone())
        host_in.copy_(host_out)
    assert torch.equal(torch.stack(seen, 1), tokens.cpu())


def test_qwen3_0_6b_decode_matches_oracle():
    """BASELINE config 2's architecture (random init, seed 0), short prompt, against the CPU oracle."""
    cfg = qwen3.Config.make(**qwen3.PRESETS["qwen3-0.6b"])
    weights = qwen3.random_init(cfg, "cuda", seed=0)
    g = torch.Generator().manual_seed(0)
    prompt = torch.randint(0, cfg.vocab_size, (1, 48), generator=g)
    steps = 4
    state = fdecode.DecodeState(weights, 1, 48, steps)
    tokens, logits = fdecode.greedy(state, prompt.cuda(), steps)
    model = omodel.Model(omodel.Config(**qwen3.PRESETS["qwen3-0.6b"]), qwen3.to_state_dict(weights))
    # teacher-force the oracle on the GPU's tokens: logits of the same prefixes
    cache = model.new_cache(1, 48 + steps)
    expect = [model.prefill(prompt, cache)]
    for step in range(steps - 1):
        expect.append(model.decode(tokens[:, step].cpu(), 48 + step, cache))
    expect = torch.stack(expect, 1).float()
    # random-init logits sit within a few bf16 ULPs of each other: allow 2e-2 of the scale as the gap
    assert_logits_close(logits.cpu(), expect, tokens.cpu(), gap=max(0.02, 2e-2 * float(expect.abs().max())))
