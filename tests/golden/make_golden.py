"""Generate the golden fixtures by running the REFERENCE's own code on CPU.

    python tests/golden/make_golden.py --reference /path/to/fast-transformer

Runs john-jpet/fast-transformer's kernel wrappers (engine/kernels/*.py) with their kernel
bodies replaced by the reference's own CPU restatements (agent/local_cpu/shim: the fake
`triton` dispatches each launch by kernel name to agent/local_cpu/shim/references.py, and
cuda_shim stands in for torch.cuda), exactly as the reference's agent/local_cpu/smoke_engine.py
does. The tiny-Qwen3 fixtures come from HF Transformers' Qwen3ForCausalLM (native greedy)
and from the reference engine itself (engine.Engine.generate over the shim).

Inputs are rebuilt from seeds by tests/golden/cases.py; each fixture stores the SHA-256 of
its inputs and the reference outputs. This script only runs where the reference source is
present; the fixtures it writes are what travels.
"""

import argparse
import contextlib
import copy
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

import torch  # noqa: E402

import cases  # noqa: E402


def setup_reference(root):
    local = os.path.join(root, "agent", "local_cpu")
    shim = os.path.join(local, "shim")
    engine = os.path.join(root, "engine")
    # Same import order as agent/local_cpu/smoke_engine.py:27-38: real torch/transformers
    # modules first, then the fake triton and the CUDA stand-ins.
    import torch._dynamo  # noqa: F401
    import torch.utils._triton
    torch.utils._triton.has_triton_package()
    torch.utils._triton.has_triton()
    import transformers.integrations.sdpa_attention  # noqa: F401
    import transformers.models.qwen3.modeling_qwen3  # noqa: F401
    from transformers import Qwen3Config, Qwen3ForCausalLM  # noqa: F401  (resolve the lazy module now)
    # torch/transformers pulled in the real triton; the reference's wrappers must see the shim.
    for name in [m for m in sys.modules if m == "triton" or m.startswith("triton.")]:
        del sys.modules[name]
    sys.path[:0] = [shim, local, engine]
    import cuda_shim
    cuda_shim.install("const", 0)
    import references  # noqa: F401  (registers the kernel references)
    import attention
    attention.sdpa_kernel = lambda *backends: contextlib.nullcontext()  # no Flash on CPU
    import kernels.decode_attention
    import kernels.linear

    def once(fn, *unused):
        fn()
        return 1.0

    kernels.linear._cold_graph_time = once
    kernels.decode_attention._graph_time = once
    return cuda_shim


def main():
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", required=True, help="checkout of john-jpet/fast-transformer")
    parser.add_argument("--only", default="")
    args = parser.parse_args()
    cuda_shim = setup_reference(args.reference)
    from kernels.argmax import argmax as ref_argmax
    from kernels.decode_attention import _attend, block_attention, decode_attention
    from kernels.merged import Split
    from kernels.qk_rope import qk_rope_cache
    from kernels.rmsnorm import add_rms_norm, embed_rms_norm, rms_norm
    from kernels.swiglu import swiglu
    import attention as ref_attention
    from types import SimpleNamespace

    only = set(args.only.split(",")) if args.only else None
    out = {}

    def want(family):
        return only is None or family in only

    with torch.inference_mode():
        if want("decode"):
            fixtures = {}
            for case in cases.DECODE_CASES:
                name = case[0]
                q, k, v, position, scale = cases.decode_inputs(case)
                batch, q_heads, _, dim = q.shape
                entry = {"digest": cases.digest(q, k, v, position)}
                if position.numel() == 1:
                    if name == "c1":
                        # BASELINE config 1 asks for 8 KV splits: the reference's own `_attend` with (64, 8, 4).
                        entry["out"] = _attend(q, k, v, position, scale, (64, 8, 4)).clone()
                    else:
                        entry["out"] = decode_attention(q, k, v, position, scale).clone()
                    # The eager path the engine falls back to: grouped SDPA with a length mask
                    # (engine/attention.py:27-39), on a NaN-free copy of the cache.
                    valid = int(position[0]) + 1
                    kk, vv = k.clone(), v.clone()
                    kk[:, :, valid:] = 0
                    vv[:, :, valid:] = 0
                    mask = (torch.arange(k.shape[2]) < valid).view(1, 1, 1, -1)
                    module = SimpleNamespace(num_key_value_groups=q_heads // k.shape[1])
                    entry["sdpa"] = ref_attention.grouped_sdpa(module, q, kk, vv, mask, scaling=scale)[0].clone()
                else:
                    # Per-row lengths: the reference's verify kernel with one token per row and
                    # chain 1 attends slots [0, position[b]] (decode_attention.py:286-294).
                    chain = torch.ones(batch, dtype=torch.int64)
                    entry["out"] = block_attention(q.reshape(batch, 1, q_heads, dim), k, v, position, scale, chain).clone()
                fixtures[name] = entry
                print("decode", name, flush=True)
            out["decode"] = fixtures

        if want("block"):
            fixtures = {}
            for case in cases.BLOCK_CASES:
                q, k, v, position, chain, scale, splits = cases.block_inputs(case)
                layout_key = None
                import kernels.decode_attention as kda
                shape = (q.device, *q.shape[:3], k.shape[1], k.shape[2], q.shape[3])
                kda._BLOCK_LAYOUTS[shape] = (128, splits, 4)  # the reference's own split tiling
                result = block_attention(q, k, v, position, scale, chain)
                fixtures[case[0]] = {"digest": cases.digest(q, k, v, position, chain), "out": result.clone()}
                print("block", case[0], flush=True)
            out["block"] = fixtures

        if want("rope"):
            fixtures = {}
            for case in cases.ROPE_CASES:
                x = cases.rope_inputs(case)
                digest = cases.digest(x["packed"], x["q_weight"], x["k_weight"], x["cos"], x["sin"], x["position"],
                                      x["keys"], x["values"], x["phases"])
                packed = x["packed"]
                if packed.dtype == torch.float32:
                    batch = x["keys"].shape[0]
                    packed = Split(packed, (batch, packed.shape[1] // batch, packed.shape[2]))
                q_norm = SimpleNamespace(weight=x["q_weight"], variance_epsilon=x["q_eps"])
                k_norm = SimpleNamespace(weight=x["k_weight"], variance_epsilon=x["k_eps"])
                keys, values = x["keys"].clone(), x["values"].clone()
                query = qk_rope_cache(packed, q_norm, k_norm, x["cos"], x["sin"], x["position"], keys, values,
                                      x["q_heads"], prefill=x["prefill"], rows=x["rows"], phases=x["phases"])
                fixtures[case[0]] = {"digest": digest, "query": query.transpose(1, 2).contiguous().clone(),
                                     "keys": keys, "values": values}
                print("rope", case[0], flush=True)
            out["rope"] = fixtures

        if want("pointwise"):
            fixtures = {}
            for case in cases.NORM_CASES:
                x, residual, weight, eps, table, ids = cases.norm_inputs(case)
                normed = rms_norm(x, weight, eps)
                added, summed = add_rms_norm(x, residual, weight, eps)
                embedded, hidden = embed_rms_norm(ids, table, weight, eps)
                fixtures[case[0]] = {"digest": cases.digest(x, residual, weight, table, ids), "rms": normed.clone(),
                                     "add": added.clone(), "sum": summed.clone(), "embed": embedded.clone(),
                                     "hidden": hidden.clone()}
            for case in cases.SWIGLU_CASES:
                packed = cases.swiglu_inputs(case)
                fixtures[case[0]] = {"digest": cases.digest(packed), "out": swiglu(packed).clone()}
            for case in cases.LINEAR_CASES:
                x, weight = cases.linear_inputs(case)
                # The reference's projection contract is F.linear's (verify_gpu.py:175-185).
                fixtures[case[0]] = {"digest": cases.digest(x, weight),
                                     "out": torch.nn.functional.linear(x, weight).clone()}
            for case in cases.ARGMAX_CASES:
                logits = cases.argmax_inputs(case)
                top = torch.zeros(logits.shape[0], dtype=torch.float32)
                ids = ref_argmax(logits, top=top)
                fixtures[case[0]] = {"digest": cases.digest(logits), "out": ids.clone(), "top": top.clone()}
            print("pointwise", flush=True)
            out["pointwise"] = fixtures

        if want("spec"):
            # The reference's speculation bookkeeping (engine/kernels/spec.py): propose,
            # within_margin, settle (exact and relaxed) and relocate, through the shim's
            # restatements (check_tree.py's emulation for _propose).
            from kernels import spec as ref_spec
            fixtures = {}
            for case in cases.SPEC_CASES:
                x = cases.spec_inputs(case)
                batch, tokens_per_row = x["history"].shape[0], x["tokens"]
                chains = torch.empty(batch, dtype=torch.int64)
                phases = torch.empty(batch, tokens_per_row, dtype=torch.int64)
                proposed = ref_spec.propose(x["history"], x["position"], tokens_per_row, x["drafts"], x["successor"],
                                            x["stale"], chains, phases)
                greedy = cases.spec_greedy(proposed, chains, x["vocab"], x["seed"])
                logits, top, margin = cases.spec_margin_inputs(case, proposed)
                within = ref_spec.within_margin(logits, proposed, top, margin)
                entry = {"digest": cases.digest(x["history"], x["position"], x["successor"], x["stale"], x["limit"]),
                         "tokens": proposed.clone(), "chains": chains.clone(), "phases": phases.clone(),
                         "greedy": greedy.clone(), "within": within[:, 1:].clone()}
                for relaxed in (False, True):
                    history, position, stale = x["history"].clone(), x["position"].clone(), x["stale"].clone()
                    result = torch.empty(batch, tokens_per_row + 1, dtype=torch.int64)
                    move_from = torch.empty(batch, dtype=torch.int64)
                    move_to = torch.empty(batch, dtype=torch.int64)
                    ref_spec.settle(proposed, greedy, position, x["limit"], history, result, move_from, move_to, chains,
                                    stale, within=within if relaxed else None)
                    entry["settle_relaxed" if relaxed else "settle"] = {
                        "result": result.clone(), "history": history.clone(), "move_from": move_from.clone(),
                        "move_to": move_to.clone(), "position": position.clone(), "stale": stale.clone()}
                fixtures[case[0]] = entry
                print("spec", case[0], flush=True)
            store, move_from, move_to = cases.relocate_inputs()
            moved = store.clone()
            ref_spec.relocate(moved, move_from, move_to)
            fixtures["relocate"] = {"digest": cases.digest(store, move_from, move_to), "store": moved}
            out["spec"] = fixtures

        if want("model"):
            from transformers import Qwen3Config, Qwen3ForCausalLM
            import decode as ref_decode
            import engine as ref_engine
            # A replayed prefill graph holds the kernels recorded with prefilling=True; the
            # fake graph re-runs the captured body, so replay it in that mode
            # (agent/local_cpu/smoke_engine.py: prefill_as_captured).
            prefill_forward = ref_decode.DecodeState.prefill_forward

            def prefill_as_captured(self):
                previous, self.cache.prefilling = self.cache.prefilling, True
                try:
                    prefill_forward(self)
                finally:
                    self.cache.prefilling = previous

            ref_decode.DecodeState.prefill_forward = prefill_as_captured
            config = Qwen3Config(**cases.TINY_QWEN3)
            config._attn_implementation = "sdpa"
            torch.manual_seed(0)
            native = Qwen3ForCausalLM(config).eval().to(dtype=torch.bfloat16)
            weights = cases.tiny_qwen3_weights()
            missing = native.load_state_dict(weights, strict=False)
            assert not [m for m in missing.missing_keys if m != "lm_head.weight"], missing
            native.tie_weights()
            fixtures = {}
            for case in cases.MODEL_CASES:
                prompt, steps = cases.model_prompt(case)
                # HF native cached greedy (agent/local_cpu/smoke_engine.py:77-86)
                result = native(input_ids=prompt, use_cache=True)
                tokens, logits = [], []
                for _ in range(steps):
                    last = result.logits[:, -1, :]
                    token = last.argmax(-1)
                    tokens.append(token.clone())
                    logits.append(last.float().clone())
                    result = native(input_ids=token[:, None], past_key_values=result.past_key_values, use_cache=True)
                # The reference engine itself (verify_gpu.py:203-206 construction).
                candidate = ref_engine.Engine.__new__(ref_engine.Engine)
                candidate.model = copy.deepcopy(native)
                ref_decode.optimize_model(candidate.model)
                candidate.state = None
                emitted = list(candidate.generate(prompt.tolist(), steps))
                fixtures[case[0]] = {"prompt": prompt, "native_tokens": torch.stack(tokens, 1),
                                     "native_logits": torch.stack(logits, 1),
                                     "engine_tokens": torch.tensor(emitted, dtype=torch.int64).T.contiguous()}
                print("model", case[0], fixtures[case[0]]["native_tokens"].tolist(),
                      fixtures[case[0]]["engine_tokens"].tolist(), flush=True)
            fixtures["weights_digest"] = cases.digest(*[weights[k] for k in sorted(weights)])
            out["model"] = fixtures

    for family, fixtures in out.items():
        path = os.path.join(HERE, f"{family}.pt")
        torch.save(fixtures, path)
        print("wrote", path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    main()
