"""Install the fused B200 ops into a Qwen3 model: the drop-in boundary.

The reference adapts a transformers ``Qwen3ForCausalLM`` by rebinding
``forward`` on module instances (server/model/patches/qwen3.py:420, the
patcher at :469-479, the loader at :482-501, reached from
server/model/hf_backend.py:16-18 and :89-97).  This module does the same, with
the same module and operator signatures, so the reference's engine and
scheduler call into libqwen3fused without a change:

* ``embed_tokens.forward(input_ids)``          -> :func:`~tinyserver_b200.embedding`
* every ``Qwen3RMSNorm.forward(hidden_states)`` (input/post-attention/final
  norms and the per-head q_norm/k_norm)        -> :func:`~tinyserver_b200.rms_norm`
* ``Qwen3DecoderLayer.forward(...)``: the post-attention residual add and
  ``post_attention_layernorm`` become one :func:`~tinyserver_b200.fused_add_rms_norm`;
  on a paged model ``Qwen3Model.forward`` also fuses each end-of-layer add
  into the next layer's input norm (or the final norm)
* ``Qwen3MLP.forward(x)``: ``act_fn(gate) * up`` -> :func:`~tinyserver_b200.silu_and_mul`
* on a paged model (one the reference's cache allocator gave ``k_cache`` /
  ``v_cache``): the attention pre-processing of the reference's patched
  forward (q_norm, k_norm, transposes, ``apply_rotary_pos_emb``, the per-token
  mapping loop and ``store_kv_cache_batched`` / per-sequence
  ``store_kv_cache``; qwen3.py:254-357) becomes ONE
  :func:`~tinyserver_b200.qk_norm_rope_store` launch per layer, with the
  block/slot mapping built on the device once per forward and shared by all
  layers; attention runs on this library's kernels with the reference's
  contracts -- paged decode (paged_attention.py:124-192) and varlen prefill
  (varlen_attention.py:145-218) -- or on any backend passed in.
* :func:`install_operator_overrides` rebinds the module-level names the
  reference imports (``apply_rotary_pos_emb`` in modeling_qwen3 and in
  server.model.patches.qwen3, ``store_kv_cache`` / ``store_kv_cache_batched``
  in server.model.patches.qwen3) for callers that keep the reference's own
  attention forward.

Every replacement runs on CUDA tensors only and raises otherwise: there is no
CPU or eager fallback.
"""

from __future__ import annotations

import sys
from dataclasses import dataclass
from typing import Any, Callable, Protocol

import torch

from ..kernels import fused as F
from ..kernels import kv_cache as KV

__all__ = ["AttentionBackend", "FusedDecodeAttention", "ReferenceAttention", "install_fused",
           "fused_qwen3_model_loader",
           "install_operator_overrides", "restore_operator_overrides", "allocate_kv_cache",
           "batch_mapping", "forget_batch_mapping"]


# ----------------------------------------------------------------------------
# module forwards
def _rms_norm_forward(norm: torch.nn.Module) -> Callable[[torch.Tensor], torch.Tensor]:
    def forward(hidden_states: torch.Tensor) -> torch.Tensor:
        # Qwen3RMSNorm.forward (modeling_qwen3.py:59-64) with the model's own
        # weight and eps; the weight must be in the activation dtype, as it is
        # for a model loaded or cast to that dtype.
        return F.rms_norm(hidden_states, norm.weight, norm.variance_epsilon)

    return forward


def _mlp_forward(mlp: torch.nn.Module) -> Callable[[torch.Tensor], torch.Tensor]:
    def forward(x: torch.Tensor) -> torch.Tensor:
        # Qwen3MLP.forward (modeling_qwen3.py:81-83)
        return mlp.down_proj(F.silu_and_mul(mlp.gate_proj(x), mlp.up_proj(x)))

    return forward


def _embedding_forward(emb: torch.nn.Embedding) -> Callable[[torch.Tensor], torch.Tensor]:
    def forward(input_ids: torch.Tensor) -> torch.Tensor:
        return F.embedding(input_ids, emb.weight)

    return forward


def _decoder_layer_forward(layer: torch.nn.Module) -> Callable[..., torch.Tensor]:
    post = layer.post_attention_layernorm

    def forward(hidden_states: torch.Tensor, attention_mask: torch.Tensor | None = None,
                position_ids: torch.Tensor | None = None, past_key_values: Any = None,
                use_cache: bool | None = False,
                position_embeddings: tuple[torch.Tensor, torch.Tensor] | None = None,
                **kwargs: Any) -> torch.Tensor:
        # Qwen3DecoderLayer.forward (modeling_qwen3.py:305-335); the add at :327
        # and the norm at :331 run as one pass.
        residual = hidden_states
        hidden_states = layer.input_layernorm(hidden_states)
        hidden_states, _ = layer.self_attn(
            hidden_states=hidden_states, attention_mask=attention_mask,
            position_ids=position_ids, past_key_values=past_key_values, use_cache=use_cache,
            position_embeddings=position_embeddings, **kwargs)
        hidden_states, residual = F.fused_add_rms_norm(hidden_states, residual, post.weight,
                                                       post.variance_epsilon)
        hidden_states = layer.mlp(hidden_states)
        return residual + hidden_states

    return forward


def _model_forward(base: torch.nn.Module, context: Callable[[], Any]) -> Callable[..., Any]:
    """Qwen3Model.forward (modeling_qwen3.py:378-437) for the paged serving path,
    with every residual add fused into the norm that follows it: the
    post-attention add into post_attention_layernorm, and the end-of-layer add
    (HF:333) into the NEXT layer's input_layernorm, or into the final norm
    after the last layer.  That removes one full read and write of the hidden
    state per layer against running the decoder layers one by one.  The
    causal masks are not built: the paged attention, like the reference's
    (qwen3.py:216-418), never reads them.  Each call first drops the batch
    mapping cached on the inference context, so the layers of this forward
    build it once from this forward's context."""
    from transformers.modeling_outputs import BaseModelOutputWithPast

    layers = list(base.layers[: base.config.num_hidden_layers])

    def forward(input_ids: torch.Tensor | None = None, attention_mask: Any = None,
                position_ids: torch.Tensor | None = None, past_key_values: Any = None,
                inputs_embeds: torch.Tensor | None = None, use_cache: bool | None = None,
                **kwargs: Any):
        if (input_ids is None) ^ (inputs_embeds is not None):
            raise ValueError("You must specify exactly one of input_ids or inputs_embeds")
        if use_cache or past_key_values is not None:
            raise ValueError("the fused paged model keeps its own paged KV cache: call it "
                             "with use_cache=False and no past_key_values")
        forget_batch_mapping(context())
        hidden = base.embed_tokens(input_ids) if inputs_embeds is None else inputs_embeds
        if position_ids is None:
            position_ids = torch.arange(hidden.shape[1], device=hidden.device).unsqueeze(0)
        position_embeddings = base.rotary_emb(hidden, position_ids)
        residual = hidden
        first = layers[0].input_layernorm
        x = F.rms_norm(hidden, first.weight, first.variance_epsilon)
        own = False  # residual is a buffer of ours (never the caller's inputs_embeds)
        for i, layer in enumerate(layers):
            x, _ = layer.self_attn(hidden_states=x, attention_mask=None,
                                   position_ids=position_ids, past_key_values=None,
                                   use_cache=False, position_embeddings=position_embeddings,
                                   **kwargs)
            post = layer.post_attention_layernorm
            x, residual = F.fused_add_rms_norm(x, residual, post.weight, post.variance_epsilon,
                                               inplace=own)
            own = True
            x = layer.mlp(x)
            nxt = layers[i + 1].input_layernorm if i + 1 < len(layers) else base.norm
            x, residual = F.fused_add_rms_norm(x, residual, nxt.weight, nxt.variance_epsilon,
                                               inplace=True)
        return BaseModelOutputWithPast(last_hidden_state=x, past_key_values=None)

    return forward


# ----------------------------------------------------------------------------
# paged attention
class AttentionBackend(Protocol):
    """The attention step that follows the fused pre-processing.

    ``prefill`` gets token-major q (T, Hq, D), k/v (T, Hkv, D) and the batch
    mapping; ``decode`` gets q (T, Hq, D) and reads K/V from the caches.  Both
    return (T, Hq * D)."""

    def prefill(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                batch: "BatchMapping", attn: torch.nn.Module) -> torch.Tensor: ...

    def decode(self, q: torch.Tensor, batch: "BatchMapping",
               attn: torch.nn.Module) -> torch.Tensor: ...


class ReferenceAttention:
    """The reference's own attention kernels, called the way its patched
    forward calls them: flash_attn_varlen_func for prefill (qwen3.py:182-214)
    and paged_attention_forward for decode (qwen3.py:388-408).  Imported from
    the reference package (``server.model.kernels``) on first use."""

    def __init__(self):
        from server.model.kernels.paged_attention import paged_attention_forward
        from server.model.kernels.varlen_attention import flash_attn_varlen_func

        self._varlen = flash_attn_varlen_func
        self._paged = paged_attention_forward

    def prefill(self, q, k, v, batch, attn):
        D = q.shape[-1]
        out = self._varlen(q, k, v, batch.cu_seqlens, batch.cu_seqlens, batch.max_seqlen,
                           batch.max_seqlen, causal=True, softmax_scale=D ** -0.5)
        return out.reshape(q.shape[0], -1)

    def decode(self, q, batch, attn):
        out = self._paged(q, attn.k_cache, attn.v_cache, batch.block_tables,
                          attn.k_cache.shape[2], batch.seq_lens)
        return out.reshape(q.shape[0], -1)


class FusedDecodeAttention:
    """Decode steps on this library's paged attention kernel
    (:func:`~tinyserver_b200.paged_attention_forward`, the reference's
    paged_attention_forward contract); prefill on ``prefill`` when given,
    else on this library's varlen kernel
    (:func:`~tinyserver_b200.flash_attn_varlen_func`, the reference's
    flash_attn_varlen_func contract)."""

    def __init__(self, prefill: AttentionBackend | None = None):
        self._prefill = prefill

    def prefill(self, q, k, v, batch, attn):
        if self._prefill is not None:
            return self._prefill.prefill(q, k, v, batch, attn)
        from ..kernels.attention import flash_attn_varlen_func

        D = q.shape[-1]
        out = flash_attn_varlen_func(q, k, v, batch.cu_seqlens, batch.cu_seqlens,
                                     batch.max_seqlen, batch.max_seqlen, causal=True,
                                     softmax_scale=D ** -0.5)
        return out.reshape(q.shape[0], -1)

    def decode(self, q, batch, attn):
        from ..kernels.attention import paged_attention_forward

        out = paged_attention_forward(q, attn.k_cache, attn.v_cache, batch.block_tables,
                                      attn.k_cache.shape[2], batch.seq_lens)
        return out.reshape(q.shape[0], -1)


@dataclass
class BatchMapping:
    """Per-forward index data, built once and shared by every layer."""

    key: tuple
    mode: str
    cu_seqlens: torch.Tensor     # (S + 1,) int32
    max_seqlen: int
    block_tables: torch.Tensor   # (S, max_blocks) int32, zero-padded (qwen3.py:388-397)
    seq_lens: torch.Tensor       # (S,) int32: position of each sequence's last token + 1
    block_mapping: torch.Tensor  # (T,) int64
    slot_mapping: torch.Tensor   # (T,) int64


def batch_mapping(ctx: Any, position_ids: torch.Tensor, block_size: int) -> BatchMapping:
    """Block/slot mapping of a batch from the reference's InferenceContext.

    Token t of sequence s at absolute position p goes to
    ``(block_table_s[p // block_size], p % block_size)``: the rule of the
    reference's per-token prefill loop (qwen3.py:296-303, where positions
    restart at 0 per sequence, prefill_helpers.py:27) and of its decode
    stores (kv_cache.py:49-58 with start_position = position_ids[0, i]).
    Built with one host->device copy of the block tables and one kernel,
    cached on the context object, so every layer of the forward reuses it.

    The cache key is the identity of ``position_ids`` (address, version,
    size) and the mode, not the sequences' contents.  The fused model forward
    drops the cache when it starts (:func:`forget_batch_mapping`), so a
    context object reused from one forward to the next is rebuilt for each.
    A caller that runs the attention layers without that model forward and
    reuses one context object must make a new context per step, as the
    reference's engine does (engine.py:579-582), or call
    :func:`forget_batch_mapping` between steps."""
    dev = position_ids.device
    key = (position_ids.data_ptr(), position_ids._version, position_ids.numel(), ctx.mode,
           block_size)
    cached = getattr(ctx, "_tinyserver_b200_mapping", None)
    if cached is not None and cached.key == key:
        return cached
    seqs = ctx.sequences
    if not seqs:
        raise ValueError("inference context has no sequences")
    lens = [int(s["num_tokens"]) for s in seqs] if ctx.mode == "prefill" else [1] * len(seqs)
    T = position_ids.numel()
    if sum(lens) != T or any(n <= 0 for n in lens):
        raise ValueError(f"{ctx.mode}: sequence lengths {lens} do not tile {T} tokens")
    max_blocks = max(len(s["block_table"]) for s in seqs)
    tables = torch.zeros(len(seqs), max(1, max_blocks), dtype=torch.int32)
    for i, s in enumerate(seqs):
        tables[i, :len(s["block_table"])] = torch.as_tensor(s["block_table"], dtype=torch.int32)
    cu = torch.zeros(len(seqs) + 1, dtype=torch.int32)
    cu[1:] = torch.cumsum(torch.tensor(lens, dtype=torch.int32), 0)
    host = torch.cat([cu, tables.view(-1)]).pin_memory()
    dev_ints = host.to(dev, non_blocking=True)
    cu_d = dev_ints[:len(seqs) + 1]
    tables_d = dev_ints[len(seqs) + 1:].view(len(seqs), -1)
    pos = position_ids.reshape(-1)
    bm, sm = F.build_slot_mapping(cu_d, pos, tables_d, block_size)
    seq_lens = (pos[cu_d[1:].long() - 1] + 1).to(torch.int32)
    m = BatchMapping(key, ctx.mode, cu_d, max(lens), tables_d, seq_lens, bm, sm)
    try:
        setattr(ctx, "_tinyserver_b200_mapping", m)
    except AttributeError:  # a context type with __slots__: rebuild per layer
        pass
    return m


def forget_batch_mapping(ctx: Any) -> None:
    """Drop the batch mapping cached on an inference context (if any)."""
    if getattr(ctx, "_tinyserver_b200_mapping", None) is not None:
        try:
            setattr(ctx, "_tinyserver_b200_mapping", None)
        except AttributeError:
            pass


def _paged_attention_forward(attn: torch.nn.Module, context: Callable[[], Any],
                             backend: AttentionBackend) -> Callable[..., Any]:
    num_q = attn.config.num_attention_heads
    num_kv = attn.config.num_key_value_heads
    D = attn.head_dim

    def forward(hidden_states: torch.Tensor,
                position_embeddings: tuple[torch.Tensor, torch.Tensor] | None = None,
                attention_mask: torch.Tensor | None = None,
                position_ids: torch.Tensor | None = None, past_key_values: Any = None,
                **kwargs: Any) -> tuple[torch.Tensor, None]:
        # Same signature and semantics as the reference's _page_attention_forward
        # (qwen3.py:216-418): one flattened batch (1, T, hidden).
        if position_ids is None:
            raise ValueError("position_ids are required by the fused paged attention forward")
        batch, seq_len, _ = hidden_states.shape
        T = batch * seq_len
        q = attn.q_proj(hidden_states).view(T, num_q, D)
        k = attn.k_proj(hidden_states).view(T, num_kv, D)
        v = attn.v_proj(hidden_states).view(T, num_kv, D)
        ctx = context()
        m = batch_mapping(ctx, position_ids, attn.k_cache.shape[2])
        qw = attn.q_norm.weight if hasattr(attn, "q_norm") else None
        kw = attn.k_norm.weight if hasattr(attn, "k_norm") else None
        eps = attn.q_norm.variance_epsilon if qw is not None else \
            (attn.k_norm.variance_epsilon if kw is not None else 0.0)
        if position_embeddings is not None:
            cos, sin = position_embeddings
            rope = dict(cos=cos.reshape(T, D), sin=sin.reshape(T, D))
        else:
            rope = dict(cos=None, sin=None, positions=position_ids.reshape(-1),
                        inv_freq=attn._tinyserver_b200_inv_freq)
        want_k = ctx.mode == "prefill"
        q_out, k_out = F.qk_norm_rope_store(
            q, k, v, qw, kw, eps, rope.pop("cos"), rope.pop("sin"), attn.k_cache, attn.v_cache,
            m.block_mapping, m.slot_mapping, want_k_out=want_k, **rope)
        if ctx.mode == "prefill":
            out = backend.prefill(q_out, k_out, v, m, attn)
        else:
            out = backend.decode(q_out, m, attn)
        return attn.o_proj(out.reshape(batch, seq_len, -1)), None

    return forward


def _reference_context() -> Callable[[], Any]:
    from server.model.inference_context import get_inference_context

    return get_inference_context


# ----------------------------------------------------------------------------
def install_fused(model: torch.nn.Module, *, paged: bool | None = None,
                  context: Callable[[], Any] | None = None,
                  attention: AttentionBackend | None = None) -> torch.nn.Module:
    """Rebind the forwards of ``model`` (a transformers Qwen3ForCausalLM or its
    ``.model``) to the fused ops, in place; returns the model.

    ``paged`` (default: whether the layers carry ``k_cache``/``v_cache``)
    also replaces each attention forward with the fused paged one, which reads
    the batch layout from ``context()`` (default: the reference's
    ``get_inference_context``) and runs ``attention`` after the fused store
    (default: this library's paged decode and varlen prefill kernels)."""
    from transformers.models.qwen3.modeling_qwen3 import (Qwen3DecoderLayer, Qwen3MLP,
                                                          Qwen3RMSNorm)

    base = model.model if hasattr(model, "model") and hasattr(model.model, "layers") else model
    for mod in base.modules():
        if isinstance(mod, Qwen3RMSNorm):
            mod.forward = _rms_norm_forward(mod)
        elif isinstance(mod, Qwen3MLP):
            act = getattr(mod.config, "hidden_act", "silu")
            if act != "silu":
                raise ValueError(f"install_fused: MLP activation {act!r} is not silu")
            mod.forward = _mlp_forward(mod)
        elif isinstance(mod, Qwen3DecoderLayer):
            mod.forward = _decoder_layer_forward(mod)
    emb = base.embed_tokens
    if emb.max_norm is not None:
        raise ValueError("install_fused: an embedding with max_norm renormalises rows")
    emb.forward = _embedding_forward(emb)

    if paged is None:
        paged = all(hasattr(layer.self_attn, "k_cache") for layer in base.layers)
    if paged:
        ctx = context or _reference_context()
        backend = attention or FusedDecodeAttention()
        inv_freq = base.rotary_emb.inv_freq
        for layer in base.layers:
            attn = layer.self_attn
            if not hasattr(attn, "k_cache"):
                raise ValueError("install_fused(paged=True): layer has no k_cache/v_cache "
                                 "(allocate the cache first)")
            attn._tinyserver_b200_inv_freq = inv_freq
            attn.forward = _paged_attention_forward(attn, ctx, backend)
        base.forward = _model_forward(base, ctx)
    return model


def allocate_kv_cache(model: torch.nn.Module, num_blocks: int, block_size: int,
                      dtype: torch.dtype, device: str | torch.device) -> torch.Tensor:
    """The reference's cache layout (qwen3.py:49-62): one zeroed
    (2, layers, num_blocks, num_kv_heads, block_size, head_dim) pool whose
    [0, i] / [1, i] views become layer i's k_cache / v_cache."""
    base = model.model if hasattr(model, "model") and hasattr(model.model, "layers") else model
    cfg = base.config
    pool = torch.zeros(2, cfg.num_hidden_layers, num_blocks, cfg.num_key_value_heads,
                       block_size, cfg.head_dim, dtype=dtype, device=device)
    for i, layer in enumerate(base.layers):
        layer.self_attn.k_cache = pool[0, i]
        layer.self_attn.v_cache = pool[1, i]
    return pool


def fused_qwen3_model_loader(model, config, memory_utilization: float, block_size: int,
                             dtype: torch.dtype, device: str) -> int:
    """Same signature and contract as the reference's ``qwen3_model_loader``
    (qwen3.py:482-501), so ``loader_by_name`` (hf_backend.py:16-18) can point
    at it: allocates the paged KV cache with the reference's allocator and
    installs the fused ops.  Returns the number of cache blocks."""
    from server.model.patches.qwen3 import qwen3_cache_allocator

    num_blocks = qwen3_cache_allocator(model, config, memory_utilization, block_size, dtype,
                                       device)
    install_fused(model, paged=True)
    return num_blocks


# ----------------------------------------------------------------------------
_saved: dict[tuple[str, str], Any] = {}


def install_operator_overrides() -> list[str]:
    """Rebind the operator names the reference imports to the fused ops (for a
    caller that keeps the reference's own attention forward).  Returns the
    names rebound; :func:`restore_operator_overrides` undoes it."""
    targets = {
        "transformers.models.qwen3.modeling_qwen3": {"apply_rotary_pos_emb":
                                                     F.apply_rotary_pos_emb},
        "server.model.patches.qwen3": {"apply_rotary_pos_emb": F.apply_rotary_pos_emb,
                                       "store_kv_cache": KV.store_kv_cache,
                                       "store_kv_cache_batched": KV.store_kv_cache_batched},
    }
    done = []
    for mod_name, names in targets.items():
        mod = sys.modules.get(mod_name)
        if mod is None:
            continue
        for name, fn in names.items():
            if hasattr(mod, name):
                _saved.setdefault((mod_name, name), getattr(mod, name))
                setattr(mod, name, fn)
                done.append(f"{mod_name}.{name}")
    return done


def restore_operator_overrides() -> None:
    for (mod_name, name), fn in list(_saved.items()):
        mod = sys.modules.get(mod_name)
        if mod is not None:
            setattr(mod, name, fn)
        del _saved[(mod_name, name)]
