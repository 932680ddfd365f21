"""Operators of the fused Qwen3 layer path (reference-compatible signatures)."""

from .fused import (apply_rotary_pos_emb, build_slot_mapping, embedding, fused_add_rms_norm,
                    qk_norm_rope_store, rms_norm, rope_cos_sin, rope_inv_freq, silu_and_mul)
from .attention import (flash_attn_varlen_func, paged_attention_forward,
                        paged_attention_workspace_bytes)
from .kv_cache import store_kv_cache, store_kv_cache_batched
from .sampling import sample_tokens, sample_tokens_seeded, uniforms_from_seeds

__all__ = ["apply_rotary_pos_emb", "build_slot_mapping", "embedding", "fused_add_rms_norm",
           "qk_norm_rope_store", "rms_norm", "rope_cos_sin", "rope_inv_freq", "silu_and_mul",
           "store_kv_cache", "store_kv_cache_batched", "paged_attention_forward",
           "paged_attention_workspace_bytes", "flash_attn_varlen_func", "sample_tokens",
           "sample_tokens_seeded", "uniforms_from_seeds"]
