"""The reference's own CPU implementation of the path, for the CPU baseline.

TEST/BENCH INFRASTRUCTURE ONLY: bench.py's CPU-baseline leg and its
``--impl reference`` arm time this; the product never imports it.

What runs is the reference's arithmetic as the reference executes it: the
transformers 5.5.0 Qwen3 modules that tinyserver's server/model calls
(``nn.Embedding``, ``Qwen3RMSNorm``, ``Qwen3RotaryEmbedding``,
``apply_rotary_pos_emb``, ``ACT2FN["silu"]``) in the order of
``Qwen3DecoderLayer.forward`` (modeling_qwen3.py:305-335) and the reference's
patched attention pre-processing (server/model/patches/qwen3.py:264-318).
The reference's KV store is a Triton GPU kernel (kv_cache.py:122-251) that
cannot run on a CPU, so the store is its torch ``index_put`` restatement:
``cache[block_mapping, :, slot_mapping, :] = k.transpose(0, 1)``.
"""

from __future__ import annotations

import torch
from torch import nn
from transformers import Qwen3Config
from transformers.activations import ACT2FN
from transformers.models.qwen3.modeling_qwen3 import (Qwen3RMSNorm, Qwen3RotaryEmbedding,
                                                      apply_rotary_pos_emb)


class ReferenceLayerPath:
    """One fused-layer step of the path with the reference's torch modules."""

    def __init__(self, shape, dtype: torch.dtype, weights: dict[str, torch.Tensor]):
        s = shape
        self.s = s
        self.dtype = dtype
        cfg = Qwen3Config(vocab_size=s.vocab, hidden_size=s.hidden,
                          intermediate_size=s.intermediate, num_attention_heads=s.num_q_heads,
                          num_key_value_heads=s.num_kv_heads, head_dim=s.head_dim,
                          rms_norm_eps=s.eps, max_position_embeddings=131072,
                          rope_parameters={"rope_type": "default", "rope_theta": s.rope_theta})
        with torch.no_grad():
            self.embed = nn.Embedding(s.vocab, s.hidden, _weight=weights["embed_weight"])
            self.input_layernorm = Qwen3RMSNorm(s.hidden, eps=s.eps).to(dtype)
            self.post_attention_layernorm = Qwen3RMSNorm(s.hidden, eps=s.eps).to(dtype)
            self.q_norm = Qwen3RMSNorm(s.head_dim, eps=s.eps).to(dtype)
            self.k_norm = Qwen3RMSNorm(s.head_dim, eps=s.eps).to(dtype)
            for name in ("input_layernorm", "post_attention_layernorm", "q_norm", "k_norm"):
                getattr(self, name).weight.copy_(weights[name])
        self.rotary_emb = Qwen3RotaryEmbedding(cfg)
        self.act_fn = ACT2FN["silu"]

    @torch.no_grad()
    def step(self, ids, positions, x_mlp, residual_unused, qkv, attn_out, gate_up, k_cache,
             v_cache, block_mapping, slot_mapping):
        s = self.s
        T = ids.shape[0]
        D, Hq, Hkv, I = s.head_dim, s.num_q_heads, s.num_kv_heads, s.intermediate
        hidden = self.embed(ids[None])                                   # HF:392
        residual = hidden
        hidden = residual + x_mlp[None]                                  # HF:333 (prev. layer)
        residual = hidden
        normed = self.input_layernorm(hidden)                            # HF:316
        cos, sin = self.rotary_emb(hidden, positions[None])              # HF:421
        q = qkv[None, :, : Hq * D].view(1, T, Hq, D)                     # qwen3.py:264
        k = qkv[None, :, Hq * D:(Hq + Hkv) * D].view(1, T, Hkv, D)
        v = qkv[None, :, (Hq + Hkv) * D:].view(1, T, Hkv, D)
        q = self.q_norm(q)                                               # qwen3.py:268-271
        k = self.k_norm(k)
        q = q.transpose(1, 2)                                            # qwen3.py:273-275
        k = k.transpose(1, 2)
        v = v.transpose(1, 2)
        q, k = apply_rotary_pos_emb(q, k, cos, sin)                      # qwen3.py:287
        k_src = k.squeeze(0).contiguous()                                # qwen3.py:312-313
        v_src = v.squeeze(0).contiguous()
        k_cache[block_mapping, :, slot_mapping, :] = k_src.transpose(0, 1)  # kv_cache.py store
        v_cache[block_mapping, :, slot_mapping, :] = v_src.transpose(0, 1)
        hidden = residual + attn_out[None]                               # HF:327
        residual = hidden
        normed2 = self.post_attention_layernorm(hidden)                  # HF:331
        act = self.act_fn(gate_up[None, :, :I]) * gate_up[None, :, I:]   # HF:82
        return normed, q, normed2, residual, act
