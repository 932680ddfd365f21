"""The reference's own GPU code, run on the same B200 as this library's kernels.

MEASUREMENT INFRASTRUCTURE ONLY: bench.py times these legs beside its own so
that each JSON line can state the speed-up over the reference on the same GPU.
The product never imports this file.

The reference (nosyndicate/tinyserver) runs unmodified, from an offline
install into ``baseline/_ref``:

    python -m pip install --no-index --no-build-isolation --no-deps \\
        --find-links /opt/wheelhouse --target baseline/_ref <reference checkout>

That directory is git-ignored (it is the reference's code, not this
project's) but travels with the tree to the GPU box.  ``TINYSERVER_REF`` may
name another directory that holds the reference's ``server`` package.

What runs, each through the reference's public function:

* the layer path: the transformers 5.5.0 Qwen3 modules that the reference's
  ``server/model`` calls (``nn.Embedding``, ``Qwen3RMSNorm``,
  ``Qwen3RotaryEmbedding``, ``apply_rotary_pos_emb``, ``ACT2FN["silu"]``) on
  CUDA tensors in ``Qwen3DecoderLayer.forward`` order, with the reference's
  patched attention pre-processing (server/model/patches/qwen3.py:264-318):
  q/k norm, transposes, RoPE, ``.contiguous()`` copies and its Triton
  ``store_kv_cache_batched`` (server/model/kernels/kv_cache.py:194-251).  The
  block/slot mappings are given on the device, as this library's step gets
  them (the reference builds them per layer in a Python loop, which is the
  caller-side row, not these ops);
* decode attention: ``paged_attention_forward`` (paged_attention.py:124-192);
* prefill attention: ``flash_attn_varlen_func`` (varlen_attention.py:145-218);
* the sampler: ``sample_tokens`` (sampling.py:118-194), torch ops on the GPU.
"""

from __future__ import annotations

import importlib
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def reference_root() -> str | None:
    """The directory that holds the reference's ``server`` package, or None."""
    for cand in (os.environ.get("TINYSERVER_REF"), os.path.join(HERE, "_ref")):
        if cand and os.path.isdir(os.path.join(cand, "server", "model")):
            return cand
    return None


def load(module: str):
    """Import one of the reference's modules (e.g. ``server.model.kernels.kv_cache``).
    Raises ImportError with the reason when the reference is not installed."""
    root = reference_root()
    if root is None:
        raise ImportError("the reference is not installed in baseline/_ref and TINYSERVER_REF "
                          "is not set")
    if root not in sys.path:
        sys.path.append(root)  # appended: it must not shadow this repository's modules
    return importlib.import_module(module)


class ReferenceGpuLayer:
    """One pass of the fused-layer path as the reference computes it on the GPU."""

    def __init__(self, shape, dtype: torch.dtype, weights: dict[str, torch.Tensor]):
        from torch import nn
        from transformers import Qwen3Config
        from transformers.activations import ACT2FN
        from transformers.models.qwen3 import modeling_qwen3 as hf

        s = self.s = shape
        dev = weights["embed_weight"].device
        cfg = Qwen3Config(vocab_size=s.vocab, hidden_size=s.hidden,
                          intermediate_size=s.intermediate, num_attention_heads=s.num_q_heads,
                          num_key_value_heads=s.num_kv_heads, head_dim=s.head_dim,
                          rms_norm_eps=s.eps, max_position_embeddings=131072,
                          rope_parameters={"rope_type": "default", "rope_theta": s.rope_theta})
        with torch.no_grad():
            self.embed = nn.Embedding(s.vocab, s.hidden, _weight=weights["embed_weight"])
            self.norms = {}
            for name, width in (("input_layernorm", s.hidden),
                                ("post_attention_layernorm", s.hidden),
                                ("q_norm", s.head_dim), ("k_norm", s.head_dim)):
                m = hf.Qwen3RMSNorm(width, eps=s.eps).to(device=dev, dtype=dtype)
                m.weight.copy_(weights[name])
                self.norms[name] = m
        self.rotary_emb = hf.Qwen3RotaryEmbedding(cfg, device=dev)
        self.apply_rotary_pos_emb = hf.apply_rotary_pos_emb
        self.act_fn = ACT2FN["silu"]
        self.store = load("server.model.kernels.kv_cache").store_kv_cache_batched

    @torch.no_grad()
    def step(self, ids, positions, x_mlp, qkv, attn_out, gate_up, k_cache, v_cache,
             block_mapping, slot_mapping):
        s = self.s
        T = ids.shape[0]
        D, Hq, Hkv, I = s.head_dim, s.num_q_heads, s.num_kv_heads, s.intermediate
        n = self.norms
        hidden = self.embed(ids[None])                                   # HF:392
        hidden = hidden + x_mlp[None]                                    # HF:333 (prev. layer)
        residual = hidden
        normed = n["input_layernorm"](hidden)                            # HF:316
        cos, sin = self.rotary_emb(hidden, positions[None])              # HF:421
        q = qkv[None, :, : Hq * D].view(1, T, Hq, D)                     # qwen3.py:264-266
        k = qkv[None, :, Hq * D:(Hq + Hkv) * D].view(1, T, Hkv, D)
        v = qkv[None, :, (Hq + Hkv) * D:].view(1, T, Hkv, D)
        q = n["q_norm"](q)                                               # qwen3.py:268-271
        k = n["k_norm"](k)
        q, k, v = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)  # qwen3.py:273-275
        q, k = self.apply_rotary_pos_emb(q, k, cos, sin)                 # qwen3.py:287
        self.store(k.squeeze(0).contiguous(), v.squeeze(0).contiguous(),  # qwen3.py:311-318
                   k_cache, v_cache, block_mapping, slot_mapping)
        hidden = residual + attn_out[None]                               # HF:327
        normed2 = n["post_attention_layernorm"](hidden)                  # HF:331
        act = self.act_fn(gate_up[None, :, :I]) * gate_up[None, :, I:]   # HF:82
        return normed, q, normed2, hidden, act


def kv_store_batched():
    """The reference's Triton ``store_kv_cache_batched``."""
    return load("server.model.kernels.kv_cache").store_kv_cache_batched


def paged_attention_forward():
    """The reference's Triton decode attention."""
    return load("server.model.kernels.paged_attention").paged_attention_forward


def flash_attn_varlen_func():
    """The reference's Triton prefill attention."""
    return load("server.model.kernels.varlen_attention").flash_attn_varlen_func


def sample_tokens():
    """The reference's batched sampler (torch ops)."""
    return load("server.model.sampling").sample_tokens
