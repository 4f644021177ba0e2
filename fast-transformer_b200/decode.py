"""Qwen3 greedy decode on B200: one CUDA graph per step over the sm_100a kernels.

The structure follows the reference engine (engine/decode.py): one graph-stable KV store
[2, L, B, Hkv, C, D] (`KVCache`, decode.py:178-213), a captured decode step
(`DecodeState.decode` :639-648 / `capture` :650-668) made of `forward_last`'s layer loop
(:216-278) - embed+norm, per layer add+norm, packed QKV projection, fused QK-norm/RoPE/KV
append, split-KV decode attention, o_proj, add+norm, packed gate/up, SwiGLU, down_proj -
then the final norm, LM head and argmax, and a device-side `position += 1`. Prefill runs
eagerly through cuBLAS and torch SDPA for the big GEMMs and prompt attention (as the
reference's prefill does, engine/layers.py:69-74), with the fused kernel writing the cache.

Tensor parallelism (by KV head, see qwen3.py): the o_proj and down_proj outputs are
reduced across ranks with one NCCL all-reduce each (fp32, inside the captured graph); every
rank then runs the same norms, LM head and argmax on identical data.
"""

import math

import torch
import torch.nn.functional as F

from kernels import _native
from kernels.argmax import argmax
from kernels.decode_attention import attend as attend_decode
from kernels.linear import linear, merge, project, splits_for, supported
from kernels.merged import Split
from kernels.qk_rope import qk_rope_cache
from kernels.rmsnorm import add_rms_norm, embed_rms_norm
from kernels.swiglu import swiglu
from kernels._native import check, lib, ptr, stream

BF16 = torch.bfloat16


class KVCache:
    """Layer-local BF16 [batch, kv_heads, capacity, head_dim] buffers in one allocation."""

    def __init__(self, layers, batch, kv_heads, capacity, head_dim, device):
        self.store = torch.zeros((2, layers, batch, kv_heads, capacity, head_dim), dtype=BF16, device=device)
        self.keys = [self.store[0, layer] for layer in range(layers)]
        self.values = [self.store[1, layer] for layer in range(layers)]

    def nbytes_valid(self, length):
        """K+V bytes of all layers for ``length`` valid slots per row."""
        _, layers, batch, kv_heads, _, dim = self.store.shape
        return 2 * layers * batch * kv_heads * length * dim * 2


def rope_tables(cfg, length, device):
    """HF Qwen3RotaryEmbedding (default rope): fp32 angles position * theta^(-2i/D), cos/sin in bf16."""
    dim = cfg.head_dim
    inv_freq = 1.0 / (cfg.rope_theta ** (torch.arange(0, dim, 2, dtype=torch.int64, device=device).float() / dim))
    freqs = torch.arange(length, device=device, dtype=torch.float32)[:, None] * inv_freq[None, :]
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos().to(BF16).contiguous(), emb.sin().to(BF16).contiguous()


class _Norm:
    """The .weight/.variance_epsilon pair the reference's qk_rope_cache signature reads."""

    __slots__ = ("weight", "variance_epsilon")

    def __init__(self, weight, eps):
        self.weight, self.variance_epsilon = weight, eps


class Communicator:
    """Sum-all-reduce over the tensor-parallel group (torch.distributed / NCCL); identity at TP 1."""

    def __init__(self, group=None, size=1):
        self.group, self.size = group, size

    def all_reduce(self, tensor):
        if self.size > 1:
            torch.distributed.all_reduce(tensor, group=self.group)
        return tensor


def _qk_rope_decode(packed, layer, eps, cos, sin, position, keys, values, q_heads):
    """fb_qk_norm_rope_append on whole cos/sin tables at the device-side position (no gather)."""
    from kernels.merged import source
    is_split = isinstance(packed, Split)
    data, splits, _, shape = source(packed)
    batch, kv_heads, capacity, dim = keys.shape
    query = torch.empty((batch, 1, q_heads, dim), device=keys.device, dtype=BF16)
    check(lib.fb_qk_norm_rope_append(
        ptr(data), splits if is_split else 0, ptr(layer.q_norm), ptr(layer.k_norm), float(eps), float(eps),
        ptr(cos), ptr(sin), ptr(position), None, ptr(query), ptr(keys), ptr(values),
        batch, 1, q_heads, kv_heads, dim, capacity, 0, 1, stream()), "fb_qk_norm_rope_append")
    return query.view(batch, q_heads, 1, dim)  # one token: token-major storage is [B, Hq, 1, D]


def _project_reduced(x, weight, comm):
    """x @ W^T summed over the TP group, as a one-slab FP32 ``Split`` for the next consumer."""
    rows = x.numel() // x.shape[-1]
    flat = x.reshape(rows, x.shape[-1])
    n, k = weight.shape
    splits = splits_for(rows, n, k, x.device)
    part = project(flat, weight, splits, out_fp32=True)
    total = part if splits == 1 else merge(part, out_fp32=True).view(1, rows, n)
    comm.all_reduce(total)
    return Split(total, (*x.shape[:-1], n))


class DecodeState:
    """KV cache, RoPE tables, device-side position and token ids, and the captured decode step.

    ``prefill(prompt)`` fills cache slots [0, T) and leaves the first greedy token in
    ``token_ids``; each ``step()`` replays the graph: one greedy token per row, written to
    ``token_ids``, KV appended at ``position``, ``position += 1``.
    """

    def __init__(self, weights, batch, prompt_length, max_new_tokens, comm=None, device="cuda"):
        self.w = weights
        self.cfg = weights.cfg
        self.comm = comm or Communicator()
        self.device = torch.device(device)
        self.batch, self.prompt_length = batch, prompt_length
        self.capacity = prompt_length + max_new_tokens
        cfg = self.cfg
        self.cache = KVCache(cfg.num_hidden_layers, batch, weights.kv_heads, self.capacity, cfg.head_dim, self.device)
        self.cos, self.sin = rope_tables(cfg, self.capacity, self.device)
        self.position = torch.full((1,), prompt_length, dtype=torch.int64, device=self.device)
        self.token_ids = torch.zeros((batch, 1), dtype=torch.int64, device=self.device)
        self.scale = 1.0 / math.sqrt(cfg.head_dim)
        self.graph = None
        self.ctas = int(lib.fb_decode_attention_ctas(batch, weights.kv_heads, self.capacity, cfg.head_dim))
        # zeroed once: the fused attention merge keeps its per-pair counters at zero between calls
        self.workspace = torch.zeros(
            int(lib.fb_decode_attention_workspace(batch, weights.q_heads, weights.kv_heads, cfg.head_dim, self.ctas)),
            dtype=torch.uint8, device=self.device)
        self.attn_out = torch.empty((batch, 1, weights.q_heads, cfg.head_dim), dtype=BF16, device=self.device)

    # ------------------------------------------------------------------ decode step
    def decode(self):
        """One greedy step for every row (the captured body)."""
        w, cfg, cache, comm = self.w, self.cfg, self.cache, self.comm
        eps = cfg.rms_norm_eps
        tp = comm.size > 1
        normalized, residual = embed_rms_norm(self.token_ids, w.embed, w.layers[0].ln1, eps)
        hidden = None
        for index, layer in enumerate(w.layers):
            if index > 0:
                normalized, residual = add_rms_norm(hidden, residual, layer.ln1, eps)
            packed = linear(normalized, layer.qkv, split_ok=True)
            query = _qk_rope_decode(packed, layer, eps, self.cos, self.sin, self.position,
                                    cache.keys[index], cache.values[index], w.q_heads)
            attention = attend_decode(query, cache.keys[index], cache.values[index], self.position, self.scale,
                                      out=self.attn_out, workspace=self.workspace, ctas=self.ctas)
            attention = attention.reshape(self.batch, 1, -1)
            if tp:
                out = _project_reduced(attention, layer.o, comm)
            else:
                out = linear(attention, layer.o, split_ok=True)
            normalized, residual = add_rms_norm(out, residual, layer.ln2, eps)
            gate_up = linear(normalized, layer.gate_up, split_ok=True)
            activated = swiglu(gate_up)
            if tp:
                hidden = _project_reduced(activated, layer.down, comm)
            else:
                hidden = linear(activated, layer.down, split_ok=True)
        normalized, _ = add_rms_norm(hidden, residual, w.final_norm, eps)
        logits = linear(normalized, w.lm_head)
        self.logits = logits
        self.token_ids.copy_(argmax(logits[:, 0, :]).unsqueeze(-1))
        self.position.add_(1)

    def capture(self, warmup=3):
        """Warm every kernel and shape choice eagerly on a side stream, then capture one step.
        The warmup steps write the slot at `position`, which every real step rewrites before
        reading it."""
        current = torch.cuda.current_stream(self.device)
        side = torch.cuda.Stream(device=self.device)
        side.wait_stream(current)
        saved_position, saved_tokens = self.position.clone(), self.token_ids.clone()
        with torch.cuda.stream(side):
            for _ in range(warmup):
                self.position.copy_(saved_position)
                self.token_ids.copy_(saved_tokens)
                self.decode()
        current.wait_stream(side)
        torch.cuda.synchronize(self.device)
        self.position.copy_(saved_position)
        self.token_ids.copy_(saved_tokens)
        self.graph = torch.cuda.CUDAGraph()
        before = _native.launches
        with torch.cuda.graph(self.graph, stream=side):
            self.decode()
        #: libfastb200 kernels one replay launches
        self.launches_per_step = _native.launches - before
        current.wait_stream(side)
        torch.cuda.synchronize(self.device)

    def step(self):
        self.graph.replay()

    def release(self):
        self.graph = None

    # ------------------------------------------------------------------ prefill (eager)
    @torch.inference_mode()
    def prefill(self, prompt):
        """Prompt ids [B, T] (T == prompt_length) on the device: cache slots [0, T), first token."""
        w, cfg, comm = self.w, self.cfg, self.comm
        eps = cfg.rms_norm_eps
        batch, length = prompt.shape
        assert batch == self.batch and length == self.prompt_length
        positions = torch.arange(length, device=self.device)
        cos, sin = self.cos[:length][None].contiguous(), self.sin[:length][None].contiguous()
        last = torch.empty((batch, 1, cfg.hidden_size), dtype=BF16, device=self.device)
        last_residual = torch.empty_like(last)
        for row in range(batch):
            ids = prompt[row:row + 1]
            normalized, residual = embed_rms_norm(ids, w.embed, w.layers[0].ln1, eps)
            hidden = None
            for index, layer in enumerate(w.layers):
                if index > 0:
                    normalized, residual = add_rms_norm(hidden, residual, layer.ln1, eps)
                keys = self.cache.keys[index][row:row + 1]
                values = self.cache.values[index][row:row + 1]
                packed = F.linear(normalized, layer.qkv)
                query = qk_rope_cache(packed, _Norm(layer.q_norm, eps), _Norm(layer.k_norm, eps), cos, sin,
                                      positions, keys, values, w.q_heads, prefill=True)
                attention = F.scaled_dot_product_attention(
                    query, keys[:, :, :length], values[:, :, :length], is_causal=True, scale=self.scale,
                    enable_gqa=True)
                attention = attention.transpose(1, 2).reshape(1, length, -1)
                out = comm.all_reduce(F.linear(attention, layer.o))
                normalized, residual = add_rms_norm(out, residual, layer.ln2, eps)
                hidden = comm.all_reduce(F.linear(swiglu(F.linear(normalized, layer.gate_up)), layer.down))
            last[row] = hidden[0, -1:]
            last_residual[row] = residual[0, -1:]
        normalized, _ = add_rms_norm(last, last_residual, w.final_norm, eps)
        logits = linear(normalized, w.lm_head)
        self.token_ids.copy_(argmax(logits[:, 0, :]).unsqueeze(-1))
        self.position.fill_(length)
        return logits[:, 0, :]

    # ------------------------------------------------------------------ host-facing step
    def step_host(self, host_in, host_out):
        """The serving call: host token ids in (pinned int64 [B]), replay, host token ids out.
        Enqueues H2D, the step and D2H on the current stream; the caller synchronises."""
        self.token_ids.view(-1).copy_(host_in, non_blocking=True)
        self.graph.replay()
        host_out.copy_(self.token_ids.view(-1), non_blocking=True)


def greedy(state, prompt, steps):
    """Prefill then ``steps`` greedy tokens (eager steps): tokens [B, steps] and fp32 logits [B, steps, V]."""
    logits = state.prefill(prompt)
    tokens, all_logits = [state.token_ids[:, 0].clone()], [logits.float()]
    for _ in range(steps - 1):
        state.decode()
        tokens.append(state.token_ids[:, 0].clone())
        all_logits.append(state.logits[:, 0, :].float())
    return torch.stack(tokens, 1), torch.stack(all_logits, 1)
