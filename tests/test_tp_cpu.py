"""Tensor parallelism by KV head, on CPU ranks (gloo, world size 2 and 4): one decode step computed
from the engine's TP shards (qwen3.from_state_dict / qwen3.random_init packing) with the
oracle's arithmetic and an fp32 all-reduce after o_proj and down_proj must reproduce the
unsharded oracle's logits; every rank must hold identical logits."""

import math
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import cases
import qwen3
from oracle import attention as oatt
from oracle import model as omodel
from oracle import pointwise as opw

F32, BF16 = torch.float32, torch.bfloat16


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def sharded_decode_step(w, token_ids, keys, values, position):
    """One decode step on this rank's shard; keys/values are this rank's [L, B, Hkv_l, C, D]."""
    cfg = w.cfg
    d, eps = cfg.head_dim, cfg.rms_norm_eps
    hq, hkv = w.q_heads, w.kv_heads
    cos, sin = omodel.rope_tables(omodel.Config(**cfg.__dict__), position + 1)
    cos, sin = cos[position], sin[position]
    hidden = w.embed[token_ids][:, None]
    residual = hidden
    normalized = opw.rms_norm(hidden, w.layers[0].ln1, eps)
    pos = torch.tensor([position])
    batch = token_ids.shape[0]
    for i, layer in enumerate(w.layers):
        if i > 0:
            normalized, residual = opw.add_rms_norm(hidden, residual, layer.ln1, eps)
        packed = opw.linear(normalized, layer.qkv)
        q, k, v = packed.split((hq * d, hkv * d, hkv * d), dim=-1)
        q = omodel.Model._rope(opw.rms_norm(q.reshape(batch, 1, hq, d), layer.q_norm, eps), cos, sin)
        k = omodel.Model._rope(opw.rms_norm(k.reshape(batch, 1, hkv, d), layer.k_norm, eps), cos, sin)
        keys[i, :, :, position] = k[:, 0]
        values[i, :, :, position] = v.reshape(batch, 1, hkv, d)[:, 0]
        attn = oatt.decode_attention(q.transpose(1, 2), keys[i], values[i], pos, 1 / math.sqrt(d))
        out = attn.reshape(batch, 1, -1).to(F32) @ layer.o.to(F32).T  # partial sum over this rank's heads
        dist.all_reduce(out)
        normalized, residual = opw.add_rms_norm(out.to(BF16), residual, layer.ln2, eps)
        gate, up = qwen3.split_gate_up(layer.gate_up)
        act = opw.swiglu(torch.cat((opw.linear(normalized, gate), opw.linear(normalized, up)), -1))
        down = act.to(F32) @ layer.down.to(F32).T
        dist.all_reduce(down)
        hidden = down.to(BF16)
    normalized, _ = opw.add_rms_norm(hidden, residual, w.final_norm, eps)
    return opw.linear(normalized, w.lm_head)[:, 0]


def _worker(rank, world, port, queue, source):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.manual_seed(0)
        if source == "tiny":
            cfg = qwen3.Config.make(**cases.TINY_QWEN3)
            state = cases.tiny_qwen3_weights()
            full = qwen3.from_state_dict(cfg, state, "cpu")
            shard = qwen3.from_state_dict(cfg, state, "cpu", rank, world)
        else:
            cfg = qwen3.Config.make(**{**qwen3.PRESETS["qwen3-0.6b"], "num_hidden_layers": 2, "vocab_size": 4096})
            full = qwen3.random_init(cfg, "cpu", seed=3)
            shard = qwen3.random_init(cfg, "cpu", seed=3, tp_rank=rank, tp_size=world)
        batch, capacity, position = 3, 40, 33
        g = torch.Generator().manual_seed(5)
        cache_shape = (cfg.num_hidden_layers, batch, cfg.num_key_value_heads, capacity, cfg.head_dim)
        keys = torch.randn(cache_shape, generator=g).to(BF16)
        values = torch.randn(cache_shape, generator=g).to(BF16)
        tokens = torch.randint(0, cfg.vocab_size, (batch,), generator=g)
        lo, hi = rank * shard.kv_heads, (rank + 1) * shard.kv_heads
        logits = sharded_decode_step(shard, tokens, keys[:, :, lo:hi].clone(), values[:, :, lo:hi].clone(), position)
        gathered = [torch.empty_like(logits) for _ in range(world)]
        dist.all_gather(gathered, logits)
        if rank == 0:
            model = omodel.Model(omodel.Config(**cfg.__dict__), qwen3.to_state_dict(full))
            expect = model.decode(tokens, position, (keys.clone(), values.clone()))
            # numpy: pickled by value (a torch tensor would travel as a file descriptor that
            # dies with this process)
            queue.put((logits.float().numpy(), expect.float().numpy(), [t.float().numpy() for t in gathered]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("source,world", [("tiny", 2), ("random_init", 2), ("random_init", 4)])
def test_tp_decode_step_matches_unsharded_oracle(source, world):
    """The tiny model has 2 KV heads (TP2 at most); the 0.6B-shaped random init has 8."""
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, queue, source)) for r in range(world)]
    for p in procs:
        p.start()
    logits, expect, gathered = queue.get(timeout=300)
    logits, expect = torch.from_numpy(logits), torch.from_numpy(expect)
    gathered = [torch.from_numpy(t) for t in gathered]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert all(torch.equal(gathered[0], t) for t in gathered[1:]), "ranks disagree"
    scale = expect.float().abs().max()
    assert (logits.float() - expect.float()).abs().max() <= 2e-2 * scale
    assert torch.equal(logits.float().argmax(-1), expect.float().argmax(-1))
