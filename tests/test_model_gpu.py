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


def _host_memory_available():
    import psutil
    free = psutil.virtual_memory().available
    try:
        limit = open("/sys/fs/cgroup/memory.max").read().strip()
        used = int(open("/sys/fs/cgroup/memory.current").read().strip())
        if limit != "max":
            free = min(free, int(limit) - used)
    except OSError:
        pass
    return free


def _config4_steps(layers, steps=2):
    """The config-4 decode step (Qwen3-8B architecture truncated to ``layers``, random init seed
    0, batch 16) over 8192 cached slots per row holding seeded N(0,1) K/V (in place of a
    prefill): ``steps`` eager greedy steps with the logits kept, then the captured graph from the
    same start. Returns (weights, first ids, eager tokens, logits list, host cache)."""
    cfg = qwen3.Config.make(**{**qwen3.PRESETS["qwen3-8b"], "num_hidden_layers": layers})
    weights = qwen3.random_init(cfg, "cuda", seed=0)
    batch, length = 16, 8192
    state = fdecode.DecodeState(weights, batch, length, steps + 2)
    state.cache.store.normal_(generator=torch.Generator(device="cuda").manual_seed(3))
    first = torch.randint(0, cfg.vocab_size, (batch, 1), generator=torch.Generator().manual_seed(3)).cuda()
    tokens, logits = [], []
    state.token_ids.copy_(first)
    state.position.fill_(length)
    for _ in range(steps):
        state.decode(keep_logits=True)
        tokens.append(state.token_ids[:, 0].clone())
        logits.append(state.logits[:, 0].float().cpu())
    tokens = torch.stack(tokens, 1)
    # the captured step from the same start (it rewrites the same slots): the same tokens
    state.token_ids.copy_(first)
    state.position.fill_(length)
    state.capture()
    replayed = []
    for _ in range(steps):
        state.step()
        replayed.append(state.token_ids[:, 0].clone())
    torch.cuda.synchronize()
    state.release()
    assert torch.equal(torch.stack(replayed, 1), tokens)
    cache = (state.cache.store[0].cpu(), state.cache.store[1].cpu())
    del state
    torch.cuda.empty_cache()
    return weights, first[:, 0].cpu(), tokens.cpu(), logits, cache


def test_qwen3_8b_layer_shapes_full_context_match_oracle():
    """Config 4's per-rank shapes at full context - batch 16, 8192 cached slots, 32/8 heads,
    hidden 4096, SwiGLU 12288, the 151936-row LM head - on the 2-layer truncation of the model
    (so no depth drift), two greedy steps, against the CPU oracle teacher-forced on the same
    cache: logits within 2e-2 of their scale and the chosen token's gap within the same."""
    weights, first, tokens, logits, cache = _config4_steps(2)
    model = omodel.Model(omodel.Config(**{**qwen3.PRESETS["qwen3-8b"], "num_hidden_layers": 2}),
                         qwen3.to_state_dict(weights))
    inputs = [first, tokens[:, 0]]
    expect = torch.stack([model.decode(inputs[s], 8192 + s, cache).float() for s in range(2)], 1)
    scale = float(expect.abs().max())
    assert_logits_close(torch.stack(logits, 1), expect, tokens, gap=max(0.02, 2e-2 * scale))


def _hf_eager_logits(state_dict, first, cache, layers):
    """The reference's own eager path on the host - HF Transformers Qwen3ForCausalLM, bf16, SDPA
    (the model the reference engine wraps) - one greedy step after ``cache``'s first 8192 slots."""
    import warnings
    from transformers import DynamicCache, Qwen3Config, Qwen3ForCausalLM
    from transformers.initialization import no_init_weights
    warnings.filterwarnings("ignore")
    cfg = Qwen3Config(**{**qwen3.PRESETS["qwen3-8b"], "num_hidden_layers": layers}, max_position_embeddings=40960)
    cfg._attn_implementation = "sdpa"
    default = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    try:
        with no_init_weights():
            model = Qwen3ForCausalLM(cfg)
    finally:
        torch.set_default_dtype(default)
    model.load_state_dict(state_dict, strict=False, assign=True)
    model.lm_head.weight = model.model.embed_tokens.weight
    model.eval()
    hf_cache = DynamicCache(config=cfg)
    for layer in range(layers):
        hf_cache.update(cache[0][layer, :, :, :8192], cache[1][layer, :, :, :8192], layer)
    with torch.inference_mode():
        return model(input_ids=first[:, None], past_key_values=hf_cache, use_cache=True).logits[:, -1].float()


def test_qwen3_8b_config4_full_size_drift_within_reference_eager():
    """BASELINE config 4 at full size, the shape bench.py times: the 36-layer Qwen3-8B
    architecture at batch 16 over 8192 cached slots per row (the persistent attention form,
    split-K projections, the fused LM-head argmax over 1187 tiles). Graph replay equals the eager
    steps. Against the CPU oracle (teacher-forced on the same cache) the logits differ by
    rounding-order drift that grows with depth in a random-init network (measured on B200: 0.9%
    of the logit scale at 2 layers, 2.1% at 8, 5.3% at 36), so the bar is the reference's own
    eager path: HF Transformers' Qwen3 in bf16 on the host, on the same weights and cache, must
    not sit closer to the oracle than the B200 step by more than a quarter (max and mean
    deviation), and the B200 step stays within 1e-1 of the scale. Needs ~80 GB of host memory."""
    if _host_memory_available() < (96 << 30):
        pytest.skip("the host cannot hold the 8B weights, the 16 x 8192-slot cache and the HF model")
    weights, first, tokens, logits, cache = _config4_steps(36)
    state_dict = qwen3.to_state_dict(weights)
    del weights
    torch.cuda.empty_cache()
    model = omodel.Model(omodel.Config(**qwen3.PRESETS["qwen3-8b"]), state_dict)
    expect = model.decode(first, 8192, (cache[0].clone(), cache[1].clone())).float()
    hf = _hf_eager_logits(state_dict, first, cache, 36)
    gpu = logits[0]
    scale = float(expect.abs().max())
    gpu_err, hf_err = (gpu - expect).abs(), (hf - expect).abs()
    print(f"config 4 step vs oracle: B200 max {gpu_err.max():.4f} mean {gpu_err.mean():.5f}; "
          f"HF eager max {hf_err.max():.4f} mean {hf_err.mean():.5f}; scale {scale:.3f}")
    assert float(gpu_err.max()) <= 1e-1 * scale
    assert float(gpu_err.max()) <= 1.25 * float(hf_err.max())
    assert float(gpu_err.mean()) <= 1.25 * float(hf_err.mean())
