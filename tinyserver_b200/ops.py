"""The path's operators as torch.library custom ops, ``torch.ops.qwen3fused.*``.

Each op calls the module-level function of the same name (the reference-
signature operators of ``tinyserver_b200.kernels``), so its arguments, checks,
errors and results are exactly those.  What the registration adds:

- the ops appear as single nodes in FX / ``torch.compile`` / ``torch.export``
  graphs instead of being traced into;
- the stores declare their in-place writes to ``k_cache`` / ``v_cache``
  (``mutates_args``), so a compiled graph orders them against the caches'
  other uses;
- every op has a fake (meta) implementation that gives the output shapes,
  dtypes and strides of the real one without launching anything, so graphs
  can be traced with fake or meta tensors.

The direct functions stay the fast path for eager callers (the model installer
uses them); these ops are for code that wants the dispatcher in the loop.
"""

import torch

from . import kernels as K

NS = "qwen3fused"

__all__ = ["NS", "OPS"]


# ---------------------------------------------------------------------------
# the fused decoder-layer ops
@torch.library.custom_op(f"{NS}::embedding", mutates_args=())
def embedding(input_ids: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    return K.embedding(input_ids, weight)


@embedding.register_fake
def _(input_ids, weight):
    return weight.new_empty(*input_ids.shape, weight.shape[1])


@torch.library.custom_op(f"{NS}::rms_norm", mutates_args=())
def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    return K.rms_norm(x, weight, eps)


@rms_norm.register_fake
def _(x, weight, eps):
    return x.new_empty(x.shape)


@torch.library.custom_op(f"{NS}::fused_add_rms_norm", mutates_args=())
def fused_add_rms_norm(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor,
                       eps: float) -> tuple[torch.Tensor, torch.Tensor]:
    return K.fused_add_rms_norm(x, residual, weight, eps)


@fused_add_rms_norm.register_fake
def _(x, residual, weight, eps):
    return x.new_empty(x.shape), x.new_empty(x.shape)


@torch.library.custom_op(f"{NS}::silu_and_mul", mutates_args=())
def silu_and_mul(gate: torch.Tensor, up: torch.Tensor | None = None) -> torch.Tensor:
    return K.silu_and_mul(gate, up)


@silu_and_mul.register_fake
def _(gate, up=None):
    if up is None:
        return gate.new_empty(*gate.shape[:-1], gate.shape[-1] // 2)
    return gate.new_empty(gate.shape)


@torch.library.custom_op(f"{NS}::rope_cos_sin", mutates_args=())
def rope_cos_sin(position_ids: torch.Tensor, inv_freq: torch.Tensor, head_dim: int,
                 dtype: torch.dtype, scaling: float = 1.0) -> tuple[torch.Tensor, torch.Tensor]:
    return K.rope_cos_sin(position_ids, inv_freq, head_dim, dtype, scaling)


@rope_cos_sin.register_fake
def _(position_ids, inv_freq, head_dim, dtype, scaling=1.0):
    shape = (*position_ids.shape, head_dim)
    return (torch.empty(shape, dtype=dtype, device=position_ids.device),
            torch.empty(shape, dtype=dtype, device=position_ids.device))


@torch.library.custom_op(f"{NS}::qk_norm_rope_store", mutates_args=("k_cache", "v_cache"))
def qk_norm_rope_store(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                       q_weight: torch.Tensor, k_weight: torch.Tensor, eps: float,
                       cos: torch.Tensor, sin: torch.Tensor, k_cache: torch.Tensor,
                       v_cache: torch.Tensor, block_mapping: torch.Tensor,
                       slot_mapping: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """q/k norm + RoPE + the paged K/V store, returning (q_out, k_out)."""
    return K.qk_norm_rope_store(q, k, v, q_weight, k_weight, eps, cos, sin, k_cache, v_cache,
                                block_mapping, slot_mapping)


@qk_norm_rope_store.register_fake
def _(q, k, v, q_weight, k_weight, eps, cos, sin, k_cache, v_cache, block_mapping,
      slot_mapping):
    T, Hq, D = q.shape
    return q.new_empty(T, Hq, D), q.new_empty(T, k.shape[1], D)


@torch.library.custom_op(f"{NS}::apply_rotary_pos_emb", mutates_args=())
def apply_rotary_pos_emb(q: torch.Tensor, k: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                         unsqueeze_dim: int = 1) -> tuple[torch.Tensor, torch.Tensor]:
    return K.apply_rotary_pos_emb(q, k, cos, sin, unsqueeze_dim)


@apply_rotary_pos_emb.register_fake
def _(q, k, cos, sin, unsqueeze_dim=1):
    # the same construction as the real op: token-major (T, H, D) rows per
    # batch entry, transposed back for unsqueeze_dim=1, then stacked
    def one(x):
        T, H = (x.shape[2], x.shape[1]) if unsqueeze_dim == 1 else (x.shape[1], x.shape[2])
        parts = []
        for _b in range(x.shape[0]):
            o = x.new_empty(T, H, x.shape[3])
            parts.append(o.transpose(0, 1) if unsqueeze_dim == 1 else o)
        return torch.stack(parts) if len(parts) > 1 else parts[0].unsqueeze(0)

    return one(q), one(k)


@torch.library.custom_op(f"{NS}::store_kv_cache_batched", mutates_args=("k_cache", "v_cache"))
def store_kv_cache_batched(k_src: torch.Tensor, v_src: torch.Tensor, k_cache: torch.Tensor,
                           v_cache: torch.Tensor, block_mapping: torch.Tensor,
                           slot_mapping: torch.Tensor) -> None:
    K.store_kv_cache_batched(k_src, v_src, k_cache, v_cache, block_mapping, slot_mapping)


@store_kv_cache_batched.register_fake
def _(k_src, v_src, k_cache, v_cache, block_mapping, slot_mapping):
    return None


@torch.library.custom_op(f"{NS}::store_kv_cache", mutates_args=("k_cache", "v_cache"))
def store_kv_cache(start_position: int, block_table: torch.Tensor, k_src: torch.Tensor,
                   v_src: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor) -> None:
    K.store_kv_cache(start_position, block_table, k_src, v_src, k_cache, v_cache)


@store_kv_cache.register_fake
def _(start_position, block_table, k_src, v_src, k_cache, v_cache):
    return None


@torch.library.custom_op(f"{NS}::build_slot_mapping", mutates_args=())
def build_slot_mapping(cu_seqlens: torch.Tensor, positions: torch.Tensor,
                       block_tables: torch.Tensor, block_size: int
                       ) -> tuple[torch.Tensor, torch.Tensor]:
    return K.build_slot_mapping(cu_seqlens, positions, block_tables, block_size)


@build_slot_mapping.register_fake
def _(cu_seqlens, positions, block_tables, block_size):
    T = positions.numel()
    return (positions.new_empty(T, dtype=torch.int64), positions.new_empty(T, dtype=torch.int64))


# ---------------------------------------------------------------------------
# decode and prefill attention, and the sampler
@torch.library.custom_op(f"{NS}::paged_attention_forward", mutates_args=())
def paged_attention_forward(query: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                            block_tables: torch.Tensor, block_size: int,
                            seq_lens: torch.Tensor) -> torch.Tensor:
    return K.paged_attention_forward(query, k_cache, v_cache, block_tables, block_size, seq_lens)


@paged_attention_forward.register_fake
def _(query, k_cache, v_cache, block_tables, block_size, seq_lens):
    return torch.empty_like(query if query.stride(2) == 1 else query.contiguous())


@torch.library.custom_op(f"{NS}::flash_attn_varlen_func", mutates_args=())
def flash_attn_varlen_func(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                           cu_seqlens_q: torch.Tensor, cu_seqlens_k: torch.Tensor,
                           max_seqlen_q: int, max_seqlen_k: int, causal: bool,
                           softmax_scale: float | None = None) -> torch.Tensor:
    return K.flash_attn_varlen_func(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q,
                                    max_seqlen_k, causal, softmax_scale)


@flash_attn_varlen_func.register_fake
def _(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k, causal,
      softmax_scale=None):
    return torch.empty_like(q if q.stride(2) == 1 else q.contiguous())


@torch.library.custom_op(f"{NS}::sample_tokens", mutates_args=())
def sample_tokens(logits: torch.Tensor, temperature: torch.Tensor, top_k: torch.Tensor,
                  top_p: torch.Tensor, uniforms: torch.Tensor) -> torch.Tensor:
    return K.sample_tokens(logits, temperature, top_k, top_p, uniforms)


@sample_tokens.register_fake
def _(logits, temperature, top_k, top_p, uniforms):
    return logits.new_empty(logits.shape[0], dtype=torch.int64)


@torch.library.custom_op(f"{NS}::sample_tokens_seeded", mutates_args=())
def sample_tokens_seeded(logits: torch.Tensor, temperature: torch.Tensor, top_k: torch.Tensor,
                         top_p: torch.Tensor, seeds: torch.Tensor,
                         steps: torch.Tensor) -> torch.Tensor:
    return K.sample_tokens_seeded(logits, temperature, top_k, top_p, seeds, steps)


@sample_tokens_seeded.register_fake
def _(logits, temperature, top_k, top_p, seeds, steps):
    return logits.new_empty(logits.shape[0], dtype=torch.int64)


@torch.library.custom_op(f"{NS}::uniforms_from_seeds", mutates_args=())
def uniforms_from_seeds(seeds: torch.Tensor, steps: torch.Tensor) -> torch.Tensor:
    return K.uniforms_from_seeds(seeds, steps, device=seeds.device)


@uniforms_from_seeds.register_fake
def _(seeds, steps):
    return seeds.new_empty(seeds.numel(), dtype=torch.float32)


OPS = ("embedding", "rms_norm", "fused_add_rms_norm", "silu_and_mul", "rope_cos_sin",
       "qk_norm_rope_store", "apply_rotary_pos_emb", "store_kv_cache_batched", "store_kv_cache",
       "build_slot_mapping", "paged_attention_forward", "flash_attn_varlen_func",
       "sample_tokens", "sample_tokens_seeded", "uniforms_from_seeds")
