"""The reference's own engine modules (engine/decode.py, layers.py, engine.py, attention.py,
speculate.py) import and bind to this package in place of their Triton ``kernels`` package.

CPU only, and only where the reference tree is mounted (skipped otherwise): the engine code is
the reference's, read from its checkout at test time, never copied here. The child process puts
this package's ``kernels`` in ``sys.modules`` first, then the reference's engine directory on
the path, so every ``from kernels.X import name`` in the engine resolves to the B200 wrappers.
Checks: every name the engine imports from ``kernels`` exists here with the reference's
parameter names (read from the reference's kernel sources with ``ast``), ``tune.knobs`` /
``pdl.self_test`` / ``linear.keep_native`` answer as the engine expects, and the reference's
``optimize_model`` packs a tiny HF Qwen3 whose layers then call the B200 kernels (which refuse
CPU tensors: there is no fallback path).
"""

import json
import os
import subprocess
import sys

import pytest

import conftest

REFERENCE_ENGINE = os.path.join(os.sep, "root", "reference", "engine")
PACKAGE = os.path.join(conftest.ROOT, "fast-transformer_b200")

CHILD = r'''
import ast, glob, inspect, json, os, sys
package, engine_dir = sys.argv[1], sys.argv[2]
sys.path.insert(0, package)
import kernels, kernels.argmax, kernels.decode_attention, kernels.linear, kernels.merged, kernels.pdl
import kernels.qk_rope, kernels.rmsnorm, kernels.spec, kernels.swiglu, kernels.tune
sys.path.remove(package)
sys.path.insert(0, engine_dir)
import decode, layers, engine, attention, speculate  # the reference's engine modules
checks = {}
checks["engine binds this package"] = all(
    os.path.dirname(inspect.getfile(fn)) == os.path.join(package, "kernels")
    for fn in (decode.decode_attention, decode.linear, decode.keep_native, decode.qk_rope_cache, decode.swiglu,
               decode.argmax, decode.greedy_tokens, decode.add_rms_norm, decode.embed_rms_norm, decode.rms_norm,
               decode.knobs, layers.block_attention, layers.linear, engine.pdl.self_test, decode.spec.propose))
# every `from kernels.X import a, b` and `kernels.spec.<fn>` / `pdl.<fn>` use in the engine
wanted = {}
for path in glob.glob(os.path.join(engine_dir, "*.py")):
    tree = ast.parse(open(path).read())
    for node in ast.walk(tree):
        if isinstance(node, ast.ImportFrom) and node.module and node.module.startswith("kernels."):
            for alias in node.names:
                wanted.setdefault(node.module, set()).add(alias.name)
        if isinstance(node, ast.Attribute) and isinstance(node.value, ast.Name) and node.value.id in ("spec", "pdl"):
            wanted.setdefault("kernels." + node.value.id, set()).add(node.attr)
missing, differ = [], []
for module, names in sorted(wanted.items()):
    ours = sys.modules[module]
    ref_src = os.path.join(engine_dir, "kernels", module.split(".")[1] + ".py")
    ref_defs = {n.name: n for n in ast.walk(ast.parse(open(ref_src).read())) if isinstance(n, ast.FunctionDef)}
    for name in sorted(names):
        if not hasattr(ours, name):
            missing.append(f"{module}.{name}")
            continue
        obj = getattr(ours, name)
        if callable(obj) and not isinstance(obj, type) and name in ref_defs:
            ref_args = [a.arg for a in ref_defs[name].args.args]
            our_args = list(inspect.signature(obj).parameters)
            if our_args[:len(ref_args)] != ref_args:
                differ.append(f"{module}.{name}: {our_args} vs {ref_args}")
checks["imported names exist"] = not missing
checks["signatures match"] = not differ
checks["knobs empty"] = kernels.tune.knobs(16) == []
checks["pick returns default"] = kernels.tune.pick(("k", 16), 4, (2, 4, 8), None) == 4
checks["pdl self_test without CUDA"] = kernels.pdl.self_test("cuda:0") is False
# the reference's optimize_model over a tiny HF Qwen3 (random init, CPU)
import torch
from transformers import Qwen3Config, Qwen3ForCausalLM
torch.manual_seed(0)
cfg = Qwen3Config(vocab_size=256, hidden_size=128, intermediate_size=256, num_hidden_layers=2,
                  num_attention_heads=4, num_key_value_heads=2, head_dim=64, tie_word_embeddings=True)
model = Qwen3ForCausalLM(cfg).to(torch.bfloat16).eval()
decode.optimize_model(model)
layer = model.model.layers[0]
checks["optimize_model packs layers"] = type(layer.self_attn).__name__ == "PackedAttention" and \
    type(layer.mlp).__name__ == "PackedMLP"
weight = layer.self_attn.qkv_weight
decode.keep_native(16, weight)
checks["keep_native routes to cuBLAS"] = bool(kernels.linear._NATIVE)
try:
    model.model.norm(torch.zeros(1, 1, 128, dtype=torch.bfloat16))
    checks["no CPU fallback"] = False
except ValueError as error:
    checks["no CPU fallback"] = "CUDA tensors only" in str(error)
print(json.dumps({"checks": checks, "missing": missing, "differ": differ}))
'''


@pytest.mark.skipif(not os.path.isdir(REFERENCE_ENGINE), reason="the reference checkout is not mounted here")
def test_reference_engine_imports_and_binds_this_package():
    proc = subprocess.run([sys.executable, "-c", CHILD, PACKAGE, REFERENCE_ENGINE], capture_output=True, text=True,
                          timeout=300, env=dict(os.environ, CUDA_VISIBLE_DEVICES=""))
    assert proc.returncode == 0, proc.stderr[-3000:]
    result = json.loads(proc.stdout.strip().splitlines()[-1])
    failed = {name: ok for name, ok in result["checks"].items() if not ok}
    assert not failed, (failed, result["missing"], result["differ"])
