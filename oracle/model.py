"""Oracle: Qwen3 greedy decode with the reference engine's cast points (CPU, TEST INFRASTRUCTURE ONLY).

Restates the reference engine's decode step (engine/decode.py:216-278 `forward_last`,
:639-648 `DecodeState.decode`) and prefill (:670-687), which keep HF Transformers' Qwen3
numerics (Qwen3RMSNorm, rotate-half RoPE with both products rounded, bf16 residual adds,
SiLU rounded before the up product) and use the reference's dense split-KV decode
attention for one-token steps (engine/layers.py:76) and causal SDPA for prefill
(engine/layers.py:69-74, engine/attention.py:15-20).

Weights are a dict keyed by HF parameter names (bf16). Pinned by tests/test_oracle_golden.py
against HF's Qwen3ForCausalLM greedy decode and the reference engine's own tokens.
"""

import math

import torch

from oracle import attention as oatt
from oracle import pointwise as opw

BF16, F32 = torch.bfloat16, torch.float32


class Config:
    def __init__(self, vocab_size, hidden_size, intermediate_size, num_hidden_layers, num_attention_heads,
                 num_key_value_heads, head_dim, rope_theta, rms_norm_eps=1e-6, tie_word_embeddings=True, **_):
        self.vocab = vocab_size
        self.hidden = hidden_size
        self.intermediate = intermediate_size
        self.layers = num_hidden_layers
        self.q_heads = num_attention_heads
        self.kv_heads = num_key_value_heads
        self.head_dim = head_dim
        self.theta = rope_theta
        self.eps = rms_norm_eps
        self.tie = tie_word_embeddings


def rope_tables(cfg, length):
    """HF Qwen3RotaryEmbedding (default rope type): fp32 angles, cos/sin cast to bf16."""
    dim = cfg.head_dim
    inv_freq = 1.0 / (cfg.theta ** (torch.arange(0, dim, 2, dtype=torch.int64).to(F32) / dim))
    positions = torch.arange(length, dtype=F32)
    freqs = positions[:, None] * inv_freq[None, :]
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos().to(BF16), emb.sin().to(BF16)


class Model:
    def __init__(self, cfg, weights):
        self.cfg = cfg
        self.w = weights
        self.lm_head = weights.get("lm_head.weight", weights["model.embed_tokens.weight"])

    def _layer(self, i, name):
        return self.w[f"model.layers.{i}.{name}"]

    def _attention_inputs(self, i, normalized):
        """q, k, v per head after projections, per-head norms (before RoPE)."""
        cfg = self.cfg
        q = opw.linear(normalized, self._layer(i, "self_attn.q_proj.weight"))
        k = opw.linear(normalized, self._layer(i, "self_attn.k_proj.weight"))
        v = opw.linear(normalized, self._layer(i, "self_attn.v_proj.weight"))
        shape = normalized.shape[:-1]
        q = opw.rms_norm(q.reshape(*shape, cfg.q_heads, cfg.head_dim), self._layer(i, "self_attn.q_norm.weight"), cfg.eps)
        k = opw.rms_norm(k.reshape(*shape, cfg.kv_heads, cfg.head_dim), self._layer(i, "self_attn.k_norm.weight"), cfg.eps)
        v = v.reshape(*shape, cfg.kv_heads, cfg.head_dim)
        return q, k, v

    @staticmethod
    def _rope(x, cos, sin):
        """HF apply_rotary_pos_emb in bf16: bf16(bf16(x*cos) + bf16(rotate_half(x)*sin))."""
        half = x.shape[-1] // 2
        rotated = torch.cat((-x[..., half:], x[..., :half]), dim=-1)
        direct = (x.to(F32) * cos.to(F32)).to(BF16)
        turn = (rotated.to(F32) * sin.to(F32)).to(BF16)
        return (direct.to(F32) + turn.to(F32)).to(BF16)

    def _mlp(self, i, normalized):
        gate = opw.linear(normalized, self._layer(i, "mlp.gate_proj.weight"))
        up = opw.linear(normalized, self._layer(i, "mlp.up_proj.weight"))
        return opw.linear(opw.swiglu(torch.cat((gate, up), dim=-1)), self._layer(i, "mlp.down_proj.weight"))

    def new_cache(self, batch, capacity):
        cfg = self.cfg
        shape = (cfg.layers, batch, cfg.kv_heads, capacity, cfg.head_dim)
        return torch.zeros(shape, dtype=BF16), torch.zeros(shape, dtype=BF16)

    def prefill(self, ids, cache):
        """Whole prompt [B, T]: writes cache slots [0, T), returns last-token logits [B, V] (bf16)."""
        cfg = self.cfg
        keys, values = cache
        batch, length = ids.shape
        cos, sin = rope_tables(cfg, length)
        hidden = self.w["model.embed_tokens.weight"][ids]
        residual = hidden
        normalized = opw.rms_norm(hidden, self._layer(0, "input_layernorm.weight"), cfg.eps)
        for i in range(cfg.layers):
            if i > 0:
                normalized, residual = opw.add_rms_norm(hidden, residual, self._layer(i, "input_layernorm.weight"), cfg.eps)
            q, k, v = self._attention_inputs(i, normalized)
            q = self._rope(q, cos[None, :, None, :], sin[None, :, None, :])
            k = self._rope(k, cos[None, :, None, :], sin[None, :, None, :])
            keys[i, :, :, :length] = k.transpose(1, 2)
            values[i, :, :, :length] = v.transpose(1, 2)
            groups = cfg.q_heads // cfg.kv_heads
            qq = q.transpose(1, 2).to(F32)
            kk = k.transpose(1, 2).to(F32).repeat_interleave(groups, dim=1)
            vv = v.transpose(1, 2).to(F32).repeat_interleave(groups, dim=1)
            attn = torch.nn.functional.scaled_dot_product_attention(
                qq, kk, vv, is_causal=True, scale=1.0 / math.sqrt(cfg.head_dim)).to(BF16)
            attn = attn.transpose(1, 2).reshape(batch, length, cfg.q_heads * cfg.head_dim)
            out = opw.linear(attn, self._layer(i, "self_attn.o_proj.weight"))
            normalized, residual = opw.add_rms_norm(out, residual, self._layer(i, "post_attention_layernorm.weight"), cfg.eps)
            hidden = self._mlp(i, normalized)
        normalized, _ = opw.add_rms_norm(hidden[:, -1:], residual[:, -1:], self.w["model.norm.weight"], cfg.eps)
        return opw.linear(normalized, self.lm_head)[:, 0]

    def decode(self, token_ids, position, cache, splits=None):
        """One step for tokens [B] at slot ``position`` (int; all rows): returns logits [B, V] (bf16)."""
        cfg = self.cfg
        keys, values = cache
        batch = token_ids.shape[0]
        cos, sin = rope_tables(cfg, position + 1)
        cos, sin = cos[position], sin[position]
        hidden = self.w["model.embed_tokens.weight"][token_ids][:, None]
        residual = hidden
        normalized = opw.rms_norm(hidden, self._layer(0, "input_layernorm.weight"), cfg.eps)
        pos = torch.tensor([position], dtype=torch.int64)
        for i in range(cfg.layers):
            if i > 0:
                normalized, residual = opw.add_rms_norm(hidden, residual, self._layer(i, "input_layernorm.weight"), cfg.eps)
            q, k, v = self._attention_inputs(i, normalized)
            q = self._rope(q, cos, sin)
            k = self._rope(k, cos, sin)
            keys[i, :, :, position] = k[:, 0]
            values[i, :, :, position] = v[:, 0]
            attn = oatt.decode_attention(q.transpose(1, 2), keys[i], values[i], pos, 1.0 / math.sqrt(cfg.head_dim),
                                         splits=splits)
            out = opw.linear(attn.reshape(batch, 1, -1), self._layer(i, "self_attn.o_proj.weight"))
            normalized, residual = opw.add_rms_norm(out, residual, self._layer(i, "post_attention_layernorm.weight"), cfg.eps)
            hidden = self._mlp(i, normalized)
        normalized, _ = opw.add_rms_norm(hidden, residual, self.w["model.norm.weight"], cfg.eps)
        return opw.linear(normalized, self.lm_head)[:, 0]

    def greedy(self, prompt, steps):
        """Prefill then ``steps`` greedy tokens: (tokens [B, steps], logits [B, steps, V] fp32)."""
        batch, length = prompt.shape
        cache = self.new_cache(batch, length + steps)
        logits = self.prefill(prompt, cache)
        tokens, all_logits = [], []
        for step in range(steps):
            token = opw.argmax(logits)
            tokens.append(token)
            all_logits.append(logits.to(F32))
            if step + 1 < steps:
                logits = self.decode(token, length + step, cache)
        return torch.stack(tokens, 1), torch.stack(all_logits, 1)
