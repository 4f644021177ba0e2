"""The speculation-bookkeeping oracle (oracle/spec.py) against fixtures produced by the
reference's own wrappers (engine/kernels/spec.py through its CPU shim). CPU only."""

import os

import torch

import cases
import conftest
from oracle import spec as ospec


def load():
    return torch.load(os.path.join(conftest.GOLDEN, "spec.pt"), weights_only=False)


def test_oracle_matches_reference_spec_fixtures():
    fx = load()
    for case in cases.SPEC_CASES:
        x = cases.spec_inputs(case)
        entry = fx[case[0]]
        assert entry["digest"] == cases.digest(x["history"], x["position"], x["successor"], x["stale"], x["limit"])
        tokens, chains, phases = ospec.propose(x["history"], x["position"], x["tokens"], x["drafts"], x["successor"],
                                               x["stale"])
        assert torch.equal(tokens, entry["tokens"]), case[0]
        assert torch.equal(chains, entry["chains"]), case[0]
        assert torch.equal(phases, entry["phases"]), case[0]
        logits, top, margin = cases.spec_margin_inputs(case, tokens)
        within = ospec.within_margin(logits, tokens, top, margin)
        assert torch.equal(within[:, 1:], entry["within"]), case[0]
        for key, flags in (("settle", None), ("settle_relaxed", within)):
            got = ospec.settle(tokens, entry["greedy"], x["position"], x["limit"], x["history"], chains, x["stale"],
                               within=flags)
            want = entry[key]
            for name, value in zip(("result", "history", "move_from", "move_to", "position", "stale"), got):
                assert torch.equal(value, want[name]), (case[0], key, name)
    store, move_from, move_to = cases.relocate_inputs()
    assert fx["relocate"]["digest"] == cases.digest(store, move_from, move_to)
    assert torch.equal(ospec.relocate(store, move_from, move_to), fx["relocate"]["store"])
