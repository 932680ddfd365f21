"""tinyserver_b200: B200 (sm_100a) kernels for the Qwen3 decoder layer's
memory-bound op path of tinyserver's server/model, behind its operator and
module signatures.

The kernels live in libqwen3fused.so (C ABI: include/qwen3fused.h), built
in-tree from tinyserver_b200/csrc.  Every op runs on CUDA tensors only and
raises otherwise; there is no CPU fallback.  The same operators are registered
as torch.library ops, ``torch.ops.qwen3fused.*`` (``tinyserver_b200.ops``).
"""

from ._capi import lib as load_library, lib_path
from ._runtime import check_errors
from . import ops, patches
from .kernels import (apply_rotary_pos_emb, build_slot_mapping, embedding, flash_attn_varlen_func,
                      fused_add_rms_norm,
                      paged_attention_forward, paged_attention_workspace_bytes,
                      qk_norm_rope_store, rms_norm, rope_cos_sin, rope_inv_freq, sample_tokens,
                      sample_tokens_seeded, silu_and_mul, store_kv_cache, store_kv_cache_batched,
                      uniforms_from_seeds)

__version__ = "0.1.0"

__all__ = ["apply_rotary_pos_emb", "build_slot_mapping", "check_errors", "embedding",
           "flash_attn_varlen_func", "ops", "patches",
           "fused_add_rms_norm", "load_library", "lib_path", "paged_attention_forward",
           "paged_attention_workspace_bytes", "qk_norm_rope_store", "rms_norm",
           "rope_cos_sin", "rope_inv_freq", "sample_tokens", "sample_tokens_seeded",
           "silu_and_mul", "store_kv_cache", "store_kv_cache_batched", "uniforms_from_seeds"]
