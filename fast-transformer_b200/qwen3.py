"""Qwen3 decoder weights for the B200 decode path: presets, seeded random init, packing and
tensor-parallel sharding by KV head.

Packing follows the reference's module swaps (engine/layers.py:23-26 QKV rows [q; k; v],
engine/layers.py:92-95 MLP rows [gate; up]), so one projection feeds the fused QK-norm/RoPE
kernel and one feeds SwiGLU; the gate/up rows are interleaved in 64-row blocks (gate block i,
then up block i) so that every 128-row tile of the fused projection+SwiGLU kernel holds the
gate and up rows of the same 64 features. Under tensor parallelism rank r of R owns KV heads
[r*Hkv/R, (r+1)*Hkv/R) and their whole GQA query groups, the matching rows of q/k/v and
gate/up, and the matching input columns of o_proj and down_proj; embeddings, norms and the
(tied) LM head are replicated.
"""

import hashlib
from dataclasses import dataclass

import torch

BF16 = torch.bfloat16

PRESETS = {
    # 28 layers, hidden 1024, 16/8 heads, D=128, SwiGLU 3072, vocab 151936, tied.
    "qwen3-0.6b": dict(vocab_size=151936, hidden_size=1024, intermediate_size=3072, num_hidden_layers=28,
                       num_attention_heads=16, num_key_value_heads=8, head_dim=128, rope_theta=1e6,
                       rms_norm_eps=1e-6, tie_word_embeddings=True),
    # 36 layers, hidden 4096, 32/8 heads, D=128, SwiGLU 12288, vocab 151936.
    "qwen3-8b": dict(vocab_size=151936, hidden_size=4096, intermediate_size=12288, num_hidden_layers=36,
                     num_attention_heads=32, num_key_value_heads=8, head_dim=128, rope_theta=1e6,
                     rms_norm_eps=1e-6, tie_word_embeddings=True),
}


@dataclass
class Config:
    vocab_size: int
    hidden_size: int
    intermediate_size: int
    num_hidden_layers: int
    num_attention_heads: int
    num_key_value_heads: int
    head_dim: int
    rope_theta: float
    rms_norm_eps: float = 1e-6
    tie_word_embeddings: bool = True
    max_position_embeddings: int = 40960

    @classmethod
    def make(cls, **kw):
        fields = cls.__dataclass_fields__
        return cls(**{k: v for k, v in kw.items() if k in fields})


@dataclass
class Layer:
    ln1: torch.Tensor       # input_layernorm [H]
    ln2: torch.Tensor       # post_attention_layernorm [H]
    qkv: torch.Tensor       # [(q_local + 2 kv_local) * D, H]
    q_norm: torch.Tensor    # [D]
    k_norm: torch.Tensor    # [D]
    o: torch.Tensor         # [H, q_local * D]
    gate_up: torch.Tensor   # [2 I_local, H]: 64-row gate/up blocks interleaved
    down: torch.Tensor      # [H, I_local]


class Weights:
    """One rank's shard of a Qwen3 decoder (all bf16, on ``device``)."""

    def __init__(self, cfg, layers, embed, final_norm, lm_head, tp_rank=0, tp_size=1):
        self.cfg, self.layers, self.embed, self.final_norm = cfg, layers, embed, final_norm
        self.lm_head = lm_head
        self.tp_rank, self.tp_size = tp_rank, tp_size
        if cfg.num_key_value_heads % tp_size or cfg.intermediate_size % tp_size:
            raise ValueError(f"tensor parallel size {tp_size} must divide the KV heads and the MLP width")
        self.kv_heads = cfg.num_key_value_heads // tp_size
        self.q_heads = cfg.num_attention_heads // tp_size
        self.intermediate = cfg.intermediate_size // tp_size
        # Vocabulary-parallel LM head: this rank's rows of the (replicated) LM head matrix when
        # the vocabulary splits into whole 8-row groups, else the whole matrix on every rank.
        vocab = lm_head.shape[0]
        if tp_size > 1 and vocab % (8 * tp_size) == 0:
            rows = vocab // tp_size
            self.vocab_base = tp_rank * rows
            self.lm_head_local = lm_head[self.vocab_base:self.vocab_base + rows]
        else:
            self.vocab_base = 0
            self.lm_head_local = lm_head

    def nbytes_per_step(self, vocab_parallel=True):
        """Weight bytes one decode step reads on this rank: every projection once and the LM
        head rows this rank projects (its vocabulary slice, or all of it)."""
        per_layer = sum(t.numel() for t in (self.layers[0].qkv, self.layers[0].o, self.layers[0].gate_up,
                                              self.layers[0].down)) * 2
        head = self.lm_head_local if vocab_parallel else self.lm_head
        return per_layer * len(self.layers) + head.numel() * 2


BLOCK = 64


def interleave_gate_up(gate, up):
    """[gate; up] rows -> 64-row blocks gate_0, up_0, gate_1, up_1, ... (I % 64 == 0)."""
    rows, cols = gate.shape
    if rows % BLOCK:
        raise ValueError(f"MLP width {rows} per rank must be a multiple of {BLOCK}")
    return torch.stack((gate.view(-1, BLOCK, cols), up.view(-1, BLOCK, cols)), dim=1).reshape(2 * rows, cols)


def split_gate_up(blocked):
    """Inverse of interleave_gate_up: (gate, up)."""
    rows, cols = blocked.shape
    view = blocked.view(-1, 2, BLOCK, cols)
    return view[:, 0].reshape(rows // 2, cols), view[:, 1].reshape(rows // 2, cols)


def _slices(cfg, tp_rank, tp_size):
    d = cfg.head_dim
    hq, hkv, inter = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.intermediate_size
    q = slice(tp_rank * hq // tp_size * d, (tp_rank + 1) * hq // tp_size * d)
    kv = slice(tp_rank * hkv // tp_size * d, (tp_rank + 1) * hkv // tp_size * d)
    mlp = slice(tp_rank * inter // tp_size, (tp_rank + 1) * inter // tp_size)
    return q, kv, mlp


def from_state_dict(cfg, state, device, tp_rank=0, tp_size=1):
    """Pack HF-named Qwen3 weights (``model.layers.{i}.self_attn.q_proj.weight`` ...) into this
    rank's shard."""
    q, kv, mlp = _slices(cfg, tp_rank, tp_size)

    def get(name):
        return state[name].to(device=device, dtype=BF16)

    layers = []
    for i in range(cfg.num_hidden_layers):
        p = f"model.layers.{i}."
        qkv = torch.cat((get(p + "self_attn.q_proj.weight")[q], get(p + "self_attn.k_proj.weight")[kv],
                         get(p + "self_attn.v_proj.weight")[kv]), dim=0).contiguous()
        gate_up = interleave_gate_up(get(p + "mlp.gate_proj.weight")[mlp], get(p + "mlp.up_proj.weight")[mlp]).contiguous()
        layers.append(Layer(
            ln1=get(p + "input_layernorm.weight"), ln2=get(p + "post_attention_layernorm.weight"), qkv=qkv,
            q_norm=get(p + "self_attn.q_norm.weight"), k_norm=get(p + "self_attn.k_norm.weight"),
            o=get(p + "self_attn.o_proj.weight")[:, q].contiguous(), gate_up=gate_up,
            down=get(p + "mlp.down_proj.weight")[:, mlp].contiguous()))
    embed = get("model.embed_tokens.weight").contiguous()
    lm_head = embed if cfg.tie_word_embeddings or "lm_head.weight" not in state else get("lm_head.weight").contiguous()
    return Weights(cfg, layers, embed, get("model.norm.weight"), lm_head, tp_rank, tp_size)


def _generator(seed, name, device):
    digest = hashlib.sha256(f"{seed}:{name}".encode()).digest()
    return torch.Generator(device=device).manual_seed(int.from_bytes(digest[:8], "little") & ((1 << 62) - 1))


def random_init(cfg, device, seed=0, tp_rank=0, tp_size=1, std=0.02):
    """BASELINE's random init: linear weights ~ N(0, std), RMSNorm and QK-norm weights = 1,
    tied embeddings. Every full tensor has its own seeded generator, so each rank's shard is
    the same slice of the same model whatever the TP size."""
    q, kv, mlp = _slices(cfg, tp_rank, tp_size)
    h, i, d = cfg.hidden_size, cfg.intermediate_size, cfg.head_dim
    hq, hkv = cfg.num_attention_heads, cfg.num_key_value_heads

    def linear(name, rows, cols):
        g = _generator(seed, name, device)
        return (torch.randn(rows, cols, device=device, generator=g) * std).to(BF16)

    ones_h = torch.ones(h, device=device, dtype=BF16)
    ones_d = torch.ones(d, device=device, dtype=BF16)
    layers = []
    for layer in range(cfg.num_hidden_layers):
        p = f"model.layers.{layer}."
        qkv = torch.cat((linear(p + "q", hq * d, h)[q], linear(p + "k", hkv * d, h)[kv],
                         linear(p + "v", hkv * d, h)[kv]), dim=0).contiguous()
        o = linear(p + "o", h, hq * d)[:, q].contiguous()
        gate_up = interleave_gate_up(linear(p + "gate", i, h)[mlp], linear(p + "up", i, h)[mlp]).contiguous()
        down = linear(p + "down", h, i)[:, mlp].contiguous()
        layers.append(Layer(ln1=ones_h, ln2=ones_h, qkv=qkv, q_norm=ones_d, k_norm=ones_d, o=o,
                            gate_up=gate_up, down=down))
    embed = linear("embed", cfg.vocab_size, h).contiguous()
    return Weights(cfg, layers, embed, ones_h, embed, tp_rank, tp_size)


def to_state_dict(weights, device="cpu"):
    """HF-named tensors of an unsharded (TP 1) ``Weights``: the inverse of ``from_state_dict``."""
    if weights.tp_size != 1:
        raise ValueError("to_state_dict needs the whole model (tp_size 1)")
    cfg = weights.cfg
    d, hq, hkv, inter = cfg.head_dim, cfg.num_attention_heads, cfg.num_key_value_heads, cfg.intermediate_size
    out = {"model.embed_tokens.weight": weights.embed.to(device), "model.norm.weight": weights.final_norm.to(device)}
    if weights.lm_head is not weights.embed:
        out["lm_head.weight"] = weights.lm_head.to(device)
    for i, layer in enumerate(weights.layers):
        p = f"model.layers.{i}."
        q, k, v = layer.qkv.to(device).split((hq * d, hkv * d, hkv * d), dim=0)
        gate, up = split_gate_up(layer.gate_up.to(device))
        out.update({
            p + "input_layernorm.weight": layer.ln1.to(device), p + "post_attention_layernorm.weight": layer.ln2.to(device),
            p + "self_attn.q_proj.weight": q, p + "self_attn.k_proj.weight": k, p + "self_attn.v_proj.weight": v,
            p + "self_attn.o_proj.weight": layer.o.to(device), p + "self_attn.q_norm.weight": layer.q_norm.to(device),
            p + "self_attn.k_norm.weight": layer.k_norm.to(device), p + "mlp.gate_proj.weight": gate,
            p + "mlp.up_proj.weight": up, p + "mlp.down_proj.weight": layer.down.to(device)})
    return out
