"""Speculation bookkeeping kernels (fb_spec_*) on B200 against the reference: bit-exact on the
fixtures the reference's own engine/kernels/spec.py produced, and against the oracle on
larger histories; graph-captured propose + settle replay the same results."""

import os

import pytest
import torch

import cases
import conftest
from oracle import spec as ospec

pytestmark = pytest.mark.gpu
DEV = "cuda"


def load():
    return torch.load(os.path.join(conftest.GOLDEN, "spec.pt"), weights_only=False)


def test_spec_kernels_match_reference_fixtures():
    from kernels import spec
    fx = load()
    for case in cases.SPEC_CASES:
        x = {k: (v.to(DEV) if torch.is_tensor(v) else v) for k, v in cases.spec_inputs(case).items()}
        entry = fx[case[0]]
        batch, count = x["history"].shape[0], x["tokens"]
        chains = torch.empty(batch, dtype=torch.int64, device=DEV)
        phases = torch.empty(batch, count, dtype=torch.int64, device=DEV)
        tokens = spec.propose(x["history"], x["position"], count, x["drafts"], x["successor"], x["stale"], chains,
                              phases)
        torch.cuda.synchronize()
        assert torch.equal(tokens.cpu(), entry["tokens"]), case[0]
        assert torch.equal(chains.cpu(), entry["chains"]), case[0]
        assert torch.equal(phases.cpu(), entry["phases"]), case[0]
        logits, top, margin = cases.spec_margin_inputs(case, entry["tokens"])
        within = spec.within_margin(logits.to(DEV), tokens, top.to(DEV), margin)
        assert torch.equal(within.cpu()[:, 1:], entry["within"]), case[0]
        greedy = entry["greedy"].to(DEV)
        for key, flags in (("settle", None), ("settle_relaxed", within)):
            history, position, stale = x["history"].clone(), x["position"].clone(), x["stale"].clone()
            result = torch.empty(batch, count + 1, dtype=torch.int64, device=DEV)
            move_from = torch.empty(batch, dtype=torch.int64, device=DEV)
            move_to = torch.empty(batch, dtype=torch.int64, device=DEV)
            spec.settle(tokens, greedy, position, x["limit"], history, result, move_from, move_to, chains, stale,
                        within=flags)
            torch.cuda.synchronize()
            want = entry[key]
            for name, value in (("result", result), ("history", history), ("move_from", move_from),
                                ("move_to", move_to), ("position", position), ("stale", stale)):
                assert torch.equal(value.cpu(), want[name]), (case[0], key, name)
    store, move_from, move_to = cases.relocate_inputs()
    moved = store.to(DEV)
    spec.relocate(moved, move_from.to(DEV), move_to.to(DEV))
    assert torch.equal(moved.cpu(), fx["relocate"]["store"])
    from kernels._native import device_error
    assert device_error() == 0


@pytest.mark.parametrize("size,batch,tokens,drafts,vocab", [(8192, 16, 16, (5, 8, 13, 14), 40),
                                                           (1000, 7, 9, (1, 3, 5, 8), 3)])
def test_spec_large_histories_match_oracle_and_replay_in_a_graph(size, batch, tokens, drafts, vocab):
    from kernels import spec
    case = ("big", batch, size, tokens, drafts, 8, vocab, size + batch)
    x = cases.spec_inputs(case)
    want_tokens, want_chains, want_phases = ospec.propose(x["history"], x["position"], tokens, drafts,
                                                          x["successor"], x["stale"])
    d = {k: (v.to(DEV) if torch.is_tensor(v) else v) for k, v in x.items()}
    chains = torch.empty(batch, dtype=torch.int64, device=DEV)
    phases = torch.empty(batch, tokens, dtype=torch.int64, device=DEV)
    got = spec.propose(d["history"], d["position"], tokens, drafts, d["successor"], d["stale"], chains, phases)
    torch.cuda.synchronize()
    assert torch.equal(got.cpu(), want_tokens) and torch.equal(chains.cpu(), want_chains)
    assert torch.equal(phases.cpu(), want_phases)
    greedy = cases.spec_greedy(want_tokens, want_chains, vocab, size).to(DEV)
    want = ospec.settle(want_tokens, greedy.cpu(), x["position"], x["limit"], x["history"], want_chains, x["stale"])
    # propose + settle captured once and replayed from the same starting state
    history, position, stale = d["history"].clone(), d["position"].clone(), d["stale"].clone()
    result = torch.empty(batch, tokens + 1, dtype=torch.int64, device=DEV)
    move_from = torch.empty(batch, dtype=torch.int64, device=DEV)
    move_to = torch.empty(batch, dtype=torch.int64, device=DEV)
    out = torch.empty(batch, tokens, dtype=torch.int64, device=DEV)

    def body():
        out.copy_(spec.propose(history, position, tokens, drafts, d["successor"], stale, chains, phases))
        spec.settle(out, greedy, position, d["limit"], history, result, move_from, move_to, chains, stale)

    body()  # warm
    graph = torch.cuda.CUDAGraph()
    history.copy_(d["history"]), position.copy_(d["position"]), stale.copy_(d["stale"])
    torch.cuda.synchronize()
    with torch.cuda.graph(graph):
        body()
    history.copy_(d["history"]), position.copy_(d["position"]), stale.copy_(d["stale"])
    graph.replay()
    torch.cuda.synchronize()
    for name, value, expect in zip(("result", "history", "move_from", "move_to", "position", "stale"),
                                   (result, history, move_from, move_to, position, stale), want):
        assert torch.equal(value.cpu(), expect), name
