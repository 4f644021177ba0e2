"""Qwen3 greedy decode on B200: one CUDA graph per step over the sm_100a kernels.

The structure follows the reference engine (engine/decode.py): one graph-stable KV store
[2, L, B, Hkv, C, D] (`KVCache`, decode.py:178-213), a captured decode step
(`DecodeState.decode` :639-648 / `capture` :650-668) made of `forward_last`'s layer loop
(:216-278) - embed+norm, per layer add+norm, packed QKV projection, fused QK-norm/RoPE/KV
append, split-KV decode attention, o_proj, add+norm, packed gate/up, SwiGLU, down_proj -
then the final norm, LM head and argmax, and a device-side `position += 1`. Prefill runs
eagerly: cuBLAS for the big GEMMs (as the reference's prefill does, engine/layers.py:69-74),
the tcgen05 causal flash kernel (fb_prefill_attention) for the prompt attention, and the
fused kernel writing the cache.

Tensor parallelism (by KV head, see qwen3.py): o_proj and down_proj write fp32 split-K
partials, summed in split order and stored, as 8-byte words carrying a flag (the decode
position + 1), into other ranks' receive buffers (torch symmetric memory, NVLink peer stores).
In the default push form (fb_allreduce_push) every rank stores its whole partial into every
rank's buffer and fb_allreduce_sum_add_rmsnorm sums the ranks in rank order and applies
add+RMSNorm; in the owner form (fb_reduce_scatter_push + fb_allreduce_add_rmsnorm) each value
goes to the rank owning its column slice, which sums the slice and shares it. No fence,
counter or barrier sits on the step's path. Every rank therefore runs the same norms, LM
head and argmax on bit-identical data. Prefill (eager, untimed) uses NCCL all-reduces.
"""

import ctypes

import math
import os

import torch
import torch.nn.functional as F

from kernels import _native
from kernels.argmax import argmax, fused_argmax
from kernels.prefill import prefill_attention
from kernels.decode_attention import attend as attend_decode
from kernels import linear as klinear
from kernels.linear import linear, swiglu_linear
from kernels.merged import Split
from kernels.qk_rope import qk_rope_cache
from kernels.rmsnorm import add_rms_norm, embed_rms_norm
from kernels.swiglu import swiglu
from kernels._native import check, lib, ptr, stream
import qwen3

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
    """The tensor-parallel group: identity at TP 1; NCCL all-reduce for prefill."""

    def __init__(self, group=None, size=1, rank=0):
        self.group, self.size, self.rank = group, size, rank

    def all_reduce(self, tensor):
        if self.size > 1:
            torch.distributed.all_reduce(tensor, group=self.group)
        return tensor


#: The step's all-reduce form: "push" (one NVLink phase: every rank pushes its whole partial to
#: every rank, each sums all ranks; fb_allreduce_push + fb_allreduce_sum_add_rmsnorm) or "owner"
#: (owner-computes reduce-scatter + all-gather, a quarter to an eighth of the volume in two
#: phases; fb_reduce_scatter_push + fb_allreduce_add_rmsnorm). Same bits on every rank in either.
#: Measured on B200 (config 4, the same box per pair): push 4282 / 6024 / 6645 tok/s at 2/4/8
#: ranks (0.09 / 0.32 / 0.60 ms of all-reduce and skew per step), owner 4080-4099 / 5593 / 6508
#: (0.28-0.31 / 0.52 / 0.65 ms).
#: FB_TP_ALLREDUCE overrides the default.
ALLREDUCE_FORM = os.environ.get("FB_TP_ALLREDUCE", "push")


class PeerBuffers:
    """The tensor-parallel all-reduce's receive regions in torch symmetric memory (plain NVLink
    peer mappings, never bound to an NVSwitch multicast object: a rank that dies while bound to
    one can fault its peers), uint64 words carrying a 32-bit flag each. The push form:
      recv [uses, world, rows, width]      every rank's fp32 partial
    the owner form:
      rs [uses, world, rows, width/world]  fp32 partials this rank receives as a slice owner
      ag [uses, rows, width/2]             summed bf16 pairs of whole rows
      ss [uses, world, chunks, rows]       each owner's sums of squares of its slice of a row, per
                                           512-column chunk of the slice
    and in both
      exchange [rows, world, 2]            the vocabulary-parallel argmax's bests
    with every rank's base address of each region."""

    def __init__(self, comm, uses, rows, width, device, form=None):
        os.environ["TORCH_SYMM_MEM_DISABLE_MULTICAST"] = "1"
        import torch.distributed._symmetric_memory as symm_mem
        world = comm.size
        self.uses, self.world, self.rows, self.width = uses, world, rows, width
        self.form = form or ALLREDUCE_FORM
        if self.form not in ("push", "owner"):
            raise ValueError(f"unknown all-reduce form {self.form!r}")

        def pad(nbytes):
            return (nbytes + 255) // 256 * 256

        if self.form == "push":
            sizes = {"recv": pad(uses * world * rows * width * 8)}
        else:
            sizes = {"rs": pad(uses * rows * width * 8), "ag": pad(uses * rows * (width // 2) * 8),
                     "ss": pad(uses * world * (-(-(width // world) // 512)) * rows * 8)}
        sizes["exchange"] = pad(rows * world * 2 * 8)
        offsets, total = {}, 0
        for name, size in sizes.items():
            offsets[name] = total
            total += size
        self.group = comm.group if comm.group is not None else torch.distributed.group.WORLD
        if hasattr(symm_mem, "enable_symm_mem_for_group"):
            try:
                symm_mem.enable_symm_mem_for_group(self.group.group_name)
            except Exception:  # noqa: BLE001 - newer torch enables groups on demand
                pass
        self.buf = symm_mem.empty(total, dtype=torch.uint8, device=device)
        handle = symm_mem.rendezvous(self.buf, self.group)
        self.handle = handle
        bases = [int(b) for b in handle.buffer_ptrs]
        local = self.buf.data_ptr()
        for name, offset in offsets.items():
            setattr(self, f"{name}_ptrs", (ctypes.c_void_p * world)(*[b + offset for b in bases]))
            setattr(self, f"{name}_local", ctypes.c_void_p(local + offset))
        self.reset()

    def reset(self):
        """Zero every region with all ranks idle (before first use and whenever the epoch, the
        decode position, may repeat a value: a new generation), then meet the other ranks so
        no push of the next step can land before the zeroing."""
        self.buf.zero_()
        torch.cuda.synchronize(self.buf.device)
        torch.distributed.barrier(group=self.group)
        torch.cuda.synchronize(self.buf.device)


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


def _qkv_rope_decode(x, layer, eps, cos, sin, position, keys, values, q_heads):
    """qkv projection (split partials when it has K splits) + QK-norm + RoPE + KV append for one
    decode token per row."""
    return _qk_rope_decode(linear(x, layer.qkv, split_ok=True), layer, eps, cos, sin, position, keys, values,
                           q_heads)


def _allreduce_add_norm(x, weight, comm, peers, use, epoch, residual, gain, eps, splits=None):
    """(normalized, summed) = add_rms_norm(all-reduce over ranks of x @ W^T, residual): the
    projection writes fp32 split partials, summed in split order and stored, flagged with
    epoch + 1, by NVLink peer stores. Push form: fb_allreduce_push stores this rank's whole
    partial into every rank's recv[use][rank] and fb_allreduce_sum_add_rmsnorm sums all ranks'
    slabs in rank order and applies add+RMSNorm. Owner form: fb_reduce_scatter_push stores each
    value only to the rank owning its column slice and fb_allreduce_add_rmsnorm has every owner
    sum its slice, add the residual and share the summed slice with every rank, which normalizes
    whole rows. ``splits`` overrides the K-split count (tests)."""
    rows = x.numel() // x.shape[-1]
    flat = x.reshape(rows, x.shape[-1]).contiguous()
    n, k = weight.shape
    width = residual.shape[-1]
    out = torch.empty_like(residual)
    summed = torch.empty_like(residual)
    if splits is None:
        splits = klinear.splits_for(rows, n, k, x.device)
    partials = klinear.project(flat, weight, klinear.SPLITS_OUT, splits)
    if peers.form == "push":
        check(lib.fb_allreduce_push(ptr(partials), splits, rows, n, comm.size, comm.rank, use, peers.recv_ptrs,
                                    ptr(epoch), stream()), "fb_allreduce_push")
        check(lib.fb_allreduce_sum_add_rmsnorm(peers.recv_local, use, peers.world, ptr(epoch), ptr(residual),
                                               ptr(gain), ptr(out), ptr(summed), rows, width, float(eps), stream()),
              "fb_allreduce_sum_add_rmsnorm")
        return out, summed
    check(lib.fb_reduce_scatter_push(ptr(partials), splits, rows, n, comm.size, comm.rank, use, peers.rs_ptrs,
                                     ptr(epoch), stream()), "fb_reduce_scatter_push")
    check(lib.fb_allreduce_add_rmsnorm(peers.rs_local, peers.ag_local, peers.ss_local, peers.ag_ptrs, peers.ss_ptrs,
                                       use, peers.world, comm.rank, ptr(epoch), ptr(residual), ptr(gain), ptr(out),
                                       ptr(summed), rows, width, float(eps), stream()), "fb_allreduce_add_rmsnorm")
    return out, summed


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
        self.peers = None
        if self.comm.size > 1:
            self.peers = PeerBuffers(self.comm, 2 * cfg.num_hidden_layers, batch, cfg.hidden_size, self.device)

    # ------------------------------------------------------------------ decode step
    def _rope_attention(self, normalized, layer, index):
        """qkv projection, QK-norm + RoPE + KV append (fb_qk_norm_rope_append), then decode
        attention (fb_decode_attention) for one layer. Fusing the norm/RoPE/append into the
        attention kernel's prologue measured slower on B200 (one TP8 rank's shard alone 2000
        against 1954 us per step): every CTA of a pair's cluster summed the qkv split partials
        of its query heads on the attention's critical path."""
        cache, w = self.cache, self.w
        keys, values = cache.keys[index], cache.values[index]
        query = _qkv_rope_decode(normalized, layer, self.cfg.rms_norm_eps, self.cos, self.sin, self.position, keys,
                                 values, w.q_heads)
        return attend_decode(query, keys, values, self.position, self.scale, out=self.attn_out,
                             workspace=self.workspace, ctas=self.ctas)

    def decode(self, keep_logits=False):
        """One greedy step for every row (the captured body).

        The greedy ids come from the fused LM-head argmax (no logits written; vocabulary-
        parallel under tensor parallelism). With ``keep_logits`` the full logits are projected
        (one K split, the fused kernel's arithmetic) into ``self.logits`` and reduced by
        argmax instead - the same ids.
        """
        w, cfg, cache, comm, peers = self.w, self.cfg, self.cache, self.comm, self.peers
        eps = cfg.rms_norm_eps
        layers = w.layers
        normalized, residual = embed_rms_norm(self.token_ids, w.embed, layers[0].ln1, eps)
        hidden = None
        for index, layer in enumerate(layers):
            if index > 0 and peers is None:
                normalized, residual = add_rms_norm(hidden, residual, layer.ln1, eps)
            attention = self._rope_attention(normalized, layer, index)
            attention = attention.reshape(self.batch, 1, -1)
            if peers is None:
                out = linear(attention, layer.o, split_ok=True)
                normalized, residual = add_rms_norm(out, residual, layer.ln2, eps)
            else:
                normalized, residual = _allreduce_add_norm(attention, layer.o, comm, peers, 2 * index, self.position,
                                                           residual, layer.ln2, eps)
            activated = swiglu_linear(normalized, layer.gate_up)
            if peers is None:
                hidden = linear(activated, layer.down, split_ok=True)
            else:
                following = layers[index + 1].ln1 if index + 1 < len(layers) else w.final_norm
                normalized, residual = _allreduce_add_norm(activated, layer.down, comm, peers, 2 * index + 1,
                                                           self.position, residual, following, eps)
        if peers is None:
            normalized, _ = add_rms_norm(hidden, residual, w.final_norm, eps)
        if keep_logits:
            rows = normalized.numel() // normalized.shape[-1]
            logits = klinear.project(normalized.reshape(rows, -1), w.lm_head, klinear.BF16_OUT, 1)
            self.logits = logits.view(self.batch, 1, -1)
            self.token_ids.copy_(argmax(logits).unsqueeze(-1))
        elif peers is not None and w.lm_head_local is not w.lm_head:
            fused_argmax(normalized, w.lm_head_local, out=self.token_ids.view(-1), index_base=w.vocab_base,
                         exchange=(comm.size, comm.rank, peers.exchange_ptrs, peers.exchange_local, self.position))
        elif w.lm_head_local is not w.lm_head:
            # one rank's shard run alone (timing only): its vocabulary slice, no candidate exchange
            fused_argmax(normalized, w.lm_head_local, out=self.token_ids.view(-1), index_base=w.vocab_base)
        else:
            fused_argmax(normalized, w.lm_head, out=self.token_ids.view(-1))
        self.position.add_(1)

    def capture(self, warmup=3):
        """Warm every kernel and shape choice eagerly on a side stream, then capture one step.
        The warmup steps write the slot at `position`, which every real step rewrites before
        reading it."""
        current = torch.cuda.current_stream(self.device)
        side = torch.cuda.Stream(device=self.device)
        # the copies are enqueued on the current stream before the side stream starts waiting
        # for it: the warm-up steps below run on the side stream and overwrite the originals
        saved_position, saved_tokens = self.position.clone(), self.token_ids.clone()
        side.wait_stream(current)
        with torch.cuda.stream(side):
            for _ in range(warmup):
                self.position.copy_(saved_position)
                self.token_ids.copy_(saved_tokens)
                self.decode()
        current.wait_stream(side)
        torch.cuda.synchronize(self.device)
        self.position.copy_(saved_position)
        self.token_ids.copy_(saved_tokens)
        if self.peers is not None:
            self.peers.reset()  # the warmup pushed words flagged with the position replayed next
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
        if self.peers is not None:
            self.peers.reset()  # a new generation replays positions an earlier one flagged
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
                attention = prefill_attention(query, keys[:, :, :length], values[:, :, :length], self.scale)
                attention = attention.reshape(1, length, -1)
                out = comm.all_reduce(F.linear(attention, layer.o))
                normalized, residual = add_rms_norm(out, residual, layer.ln2, eps)
                gate, up = qwen3.split_gate_up(layer.gate_up)
                hidden = comm.all_reduce(F.linear(swiglu(torch.cat((F.linear(normalized, gate),
                                                                      F.linear(normalized, up)), -1)), layer.down))
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
        state.decode(keep_logits=True)
        tokens.append(state.token_ids[:, 0].clone())
        all_logits.append(state.logits[:, 0, :].float())
    return torch.stack(tokens, 1), torch.stack(all_logits, 1)
