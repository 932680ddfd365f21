"""Functional API of the fused Qwen3 layer ops (CUDA only, no fallback).

Each function replaces one piece of the reference's eager path and matches its
rounding (fp32 math, results rounded to the tensor dtype where torch rounds):

* :func:`embedding`           -- ``nn.Embedding`` forward (modeling_qwen3.py:392)
* :func:`rms_norm`            -- ``Qwen3RMSNorm.forward`` (modeling_qwen3.py:59-64)
* :func:`fused_add_rms_norm`  -- residual add (modeling_qwen3.py:327/333) + RMSNorm
* :func:`rope_cos_sin`        -- ``Qwen3RotaryEmbedding.forward`` (modeling_qwen3.py:137-148)
* :func:`apply_rotary_pos_emb` -- same signature as modeling_qwen3.py:159
* :func:`qk_norm_rope_store`  -- q_norm/k_norm + RoPE + paged store, as
  server/model/patches/qwen3.py:268-318 chains them
* :func:`silu_and_mul`        -- ``act_fn(gate) * up`` of ``Qwen3MLP`` (modeling_qwen3.py:82)
* :func:`build_slot_mapping`  -- device-side block/slot mapping (replaces the
  per-token loop at qwen3.py:296-310)
"""

from __future__ import annotations

import ctypes

import torch

from .. import _capi
from .._runtime import (after_op, dtype_tag, index_tag, on_device, require_cuda, status_word,
                        stream_ptr)

__all__ = ["embedding", "rms_norm", "fused_add_rms_norm", "rope_cos_sin", "rope_inv_freq",
           "apply_rotary_pos_emb", "qk_norm_rope_store", "silu_and_mul", "build_slot_mapping"]


def _rows(x: torch.Tensor) -> torch.Tensor:
    """(..., H) -> (R, H) view with unit stride in H (copy only if needed)."""
    H = x.shape[-1]
    if x.stride(-1) != 1:
        x = x.contiguous()
    try:
        return x.view(-1, H)
    except RuntimeError:
        return x.contiguous().view(-1, H)


# ----------------------------------------------------------------------------
def embedding(input_ids: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """``weight[input_ids]``: bit-exact rows, shape ``input_ids.shape + (H,)``."""
    if weight.dim() != 2:
        raise ValueError(f"embedding weight must be 2D, got {tuple(weight.shape)}")
    itag = index_tag(input_ids, "embedding input_ids")
    dev = require_cuda("embedding", input_ids, weight)
    ids = input_ids.reshape(-1).contiguous()
    V, H = weight.shape
    if weight.stride(1) != 1:
        weight = weight.contiguous()
    out = torch.empty(ids.numel(), H, dtype=weight.dtype, device=dev)
    with on_device(dev):
        rc = _capi.lib().qf_embedding(ids.data_ptr(), itag, weight.data_ptr(), V, weight.stride(0),
                                      out.data_ptr(), H, ids.numel(), H, weight.element_size(),
                                      status_word(dev).data_ptr(), stream_ptr(dev))
    _capi.check(rc, "embedding")
    after_op(dev)
    return out.view(*input_ids.shape, H)


# ----------------------------------------------------------------------------
def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float,
             out: torch.Tensor | None = None) -> torch.Tensor:
    """Qwen3RMSNorm over the last dim; x and weight in the same dtype."""
    if weight.dtype != x.dtype:
        raise ValueError(f"rms_norm: weight dtype {weight.dtype} != input dtype {x.dtype}")
    if weight.dim() != 1 or weight.shape[0] != x.shape[-1]:
        raise ValueError(f"rms_norm: weight shape {tuple(weight.shape)} != ({x.shape[-1]},)")
    tag = dtype_tag(x, "rms_norm")
    dev = require_cuda("rms_norm", x, weight, out)
    x2 = _rows(x)
    y = torch.empty(x.shape, dtype=x.dtype, device=dev) if out is None else out
    y2 = _rows(y)
    if y2.data_ptr() != y.data_ptr() and out is not None:
        raise ValueError("rms_norm: out must be viewable as rows")
    w = weight.contiguous()
    with on_device(dev):
        rc = _capi.lib().qf_rmsnorm(x2.data_ptr(), x2.stride(0), w.data_ptr(), y2.data_ptr(),
                                    y2.stride(0), x2.shape[0], x2.shape[1], float(eps), tag,
                                    stream_ptr(dev))
    _capi.check(rc, "rms_norm")
    return y


def fused_add_rms_norm(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor,
                       eps: float, inplace: bool = False
                       ) -> tuple[torch.Tensor, torch.Tensor]:
    """``h = residual + x; return rms_norm(h), h`` in one pass.

    With ``inplace=True`` the new residual is written into ``residual`` (the
    returned h is that tensor)."""
    if x.shape != residual.shape:
        raise ValueError(f"fused_add_rms_norm: x {tuple(x.shape)} vs residual "
                         f"{tuple(residual.shape)}")
    if not (x.dtype == residual.dtype == weight.dtype):
        raise ValueError("fused_add_rms_norm: x, residual and weight must share a dtype")
    if weight.dim() != 1 or weight.shape[0] != x.shape[-1]:
        raise ValueError(f"fused_add_rms_norm: weight shape {tuple(weight.shape)}")
    tag = dtype_tag(x, "fused_add_rms_norm")
    dev = require_cuda("fused_add_rms_norm", x, residual, weight)
    x2 = _rows(x)
    r2 = _rows(residual)
    if inplace:
        if r2.data_ptr() != residual.data_ptr() or not residual.is_contiguous():
            raise ValueError("fused_add_rms_norm(inplace=True) needs a contiguous residual")
        h = residual
    else:
        h = torch.empty(x.shape, dtype=x.dtype, device=dev)
    h2 = h.view(-1, x.shape[-1])
    y = torch.empty(x.shape, dtype=x.dtype, device=dev)
    y2 = y.view(-1, x.shape[-1])
    w = weight.contiguous()
    with on_device(dev):
        rc = _capi.lib().qf_add_rmsnorm(x2.data_ptr(), x2.stride(0), r2.data_ptr(), r2.stride(0),
                                        w.data_ptr(), h2.data_ptr(), h2.stride(0), y2.data_ptr(),
                                        y2.stride(0), x2.shape[0], x2.shape[1], float(eps), tag,
                                        stream_ptr(dev))
    _capi.check(rc, "fused_add_rms_norm")
    return y, h


# ----------------------------------------------------------------------------
def rope_inv_freq(head_dim: int, theta: float, device=None) -> torch.Tensor:
    """inv_freq exactly as transformers' compute_default_rope_parameters builds
    it (modeling_qwen3.py:125-132): computed on the CPU in fp32, then moved."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).to(dtype=torch.float)
                           / head_dim))
    return inv.to(device) if device is not None else inv


def rope_cos_sin(position_ids: torch.Tensor, inv_freq: torch.Tensor, head_dim: int,
                 dtype: torch.dtype, scaling: float = 1.0
                 ) -> tuple[torch.Tensor, torch.Tensor]:
    """cos/sin tables of shape ``position_ids.shape + (head_dim,)`` in ``dtype``
    (Qwen3RotaryEmbedding.forward, default rope type).

    ``inv_freq`` may be any floating dtype: like the reference forward
    (``self.inv_freq[None, :, None].float()``, modeling_qwen3.py:137) it is
    upcast to float32 first, so a model cast with ``.to(bfloat16)`` (which
    also casts the inv_freq buffer) gets the same tables as under HF."""
    itag = index_tag(position_ids, "rope_cos_sin position_ids")
    dev = require_cuda("rope_cos_sin", position_ids, inv_freq)
    if not inv_freq.is_floating_point() or inv_freq.numel() != head_dim // 2:
        raise ValueError("rope_cos_sin: inv_freq must be floating with head_dim/2 entries")
    pos = position_ids.reshape(-1).contiguous()
    inv = inv_freq.to(torch.float32).contiguous()
    cos = torch.empty(*position_ids.shape, head_dim, dtype=dtype, device=dev)
    sin = torch.empty_like(cos)
    with on_device(dev):
        rc = _capi.lib().qf_rope_cos_sin(pos.data_ptr(), itag, inv.data_ptr(), pos.numel(),
                                         head_dim, float(scaling), _dtype_of(dtype), cos.data_ptr(),
                                         sin.data_ptr(), stream_ptr(dev))
    _capi.check(rc, "rope_cos_sin")
    return cos, sin


def _dtype_of(dtype: torch.dtype) -> int:
    return dtype_tag(torch.empty(0, dtype=dtype), "dtype")


def _heads_view(x: torch.Tensor, what: str) -> tuple[int, int]:
    """(token stride, head stride) of a (T, H, D) view with unit stride in D."""
    if x.dim() != 3 or x.stride(2) != 1:
        raise ValueError(f"{what}: expected a (tokens, heads, head_dim) view with contiguous "
                         f"head_dim, got shape {tuple(x.shape)} strides {x.stride()}")
    return x.stride(0), x.stride(1)


def qk_norm_rope_store(
    q: torch.Tensor, k: torch.Tensor, v: torch.Tensor | None,
    q_weight: torch.Tensor | None, k_weight: torch.Tensor | None, eps: float,
    cos: torch.Tensor | None, sin: torch.Tensor | None,
    k_cache: torch.Tensor | None = None, v_cache: torch.Tensor | None = None,
    block_mapping: torch.Tensor | None = None, slot_mapping: torch.Tensor | None = None,
    *, positions: torch.Tensor | None = None, inv_freq: torch.Tensor | None = None,
    want_k_out: bool = True, q_out: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor | None]:
    """One pass of q_norm/k_norm + neox RoPE + paged KV store.

    q: (T, Hq, D), k/v: (T, Hkv, D) views (e.g. of the projection outputs);
    cos/sin: (T, D) tables, or None with ``positions``/``inv_freq`` to compute
    them in-kernel.  Returns ``(q_out (T, Hq, D), k_out (T, Hkv, D) or None)``;
    with caches given, the rotated K and V rows go to
    ``cache[block_mapping[t], h, slot_mapping[t], :]``.
    """
    T, Hq, D = q.shape
    if k.shape[0] != T or k.shape[2] != D:
        raise ValueError(f"qk_norm_rope_store: q {tuple(q.shape)} vs k {tuple(k.shape)}")
    Hkv = k.shape[1]
    tag = dtype_tag(q, "qk_norm_rope_store")
    for t in (k, v, q_weight, k_weight, cos, sin, k_cache, v_cache):
        if t is not None and t.dtype != q.dtype:
            raise ValueError(f"qk_norm_rope_store: dtype mismatch ({t.dtype} vs {q.dtype})")
    dev = require_cuda("qk_norm_rope_store", q, k, v, q_weight, k_weight, cos, sin, k_cache,
                       v_cache, block_mapping, slot_mapping, positions, inv_freq)
    a = _capi.QkNormRopeArgs()
    a.q = q.data_ptr()
    a.q_stride_token, a.q_stride_head = _heads_view(q, "q")
    a.k = k.data_ptr()
    a.k_stride_token, a.k_stride_head = _heads_view(k, "k")
    keep = [q_weight, k_weight]  # contiguous copies stay referenced until the launch
    if q_weight is not None:
        keep[0] = q_weight.contiguous()
        a.q_weight = keep[0].data_ptr()
    if k_weight is not None:
        keep[1] = k_weight.contiguous()
        a.k_weight = keep[1].data_ptr()
    a.eps = float(eps)
    if cos is not None:
        if sin is None or cos.shape[-1] != D or sin.shape != cos.shape:
            raise ValueError("qk_norm_rope_store: cos/sin must both be (T, head_dim)")
        cos2 = cos.reshape(-1, D)
        sin2 = sin.reshape(-1, D)
        if cos2.shape[0] != T:
            raise ValueError(f"qk_norm_rope_store: cos has {cos2.shape[0]} rows for {T} tokens")
        if cos2.stride(1) != 1 or sin2.stride() != cos2.stride():
            cos2, sin2 = cos2.contiguous(), sin2.contiguous()
        keep += [cos2, sin2]
        a.cos, a.sin, a.cos_sin_token_stride = cos2.data_ptr(), sin2.data_ptr(), cos2.stride(0)
    else:
        if positions is None or inv_freq is None:
            raise ValueError("qk_norm_rope_store: give cos/sin or positions + inv_freq")
        pos = positions.reshape(-1).contiguous()
        inv = inv_freq.to(torch.float32).contiguous()
        keep += [pos, inv]
        a.positions, a.positions_type = pos.data_ptr(), index_tag(pos, "positions")
        a.inv_freq = inv.data_ptr()
    if q_out is None:
        q_out = torch.empty(T, Hq, D, dtype=q.dtype, device=dev)
    a.q_out = q_out.data_ptr()
    a.q_out_stride_token, a.q_out_stride_head = _heads_view(q_out, "q_out")
    k_out = torch.empty(T, Hkv, D, dtype=q.dtype, device=dev) if want_k_out else None
    if k_out is not None:
        a.k_out = k_out.data_ptr()
        a.k_out_stride_token, a.k_out_stride_head = Hkv * D, D
    if k_cache is not None:
        if v is None or v_cache is None or block_mapping is None or slot_mapping is None:
            raise ValueError("qk_norm_rope_store: a store needs v, v_cache and both mappings")
        if v.shape != k.shape:
            raise ValueError(f"qk_norm_rope_store: v {tuple(v.shape)} vs k {tuple(k.shape)}")
        if k_cache.dim() != 4 or k_cache.shape != v_cache.shape or \
                k_cache.shape[1] != Hkv or k_cache.shape[3] != D:
            raise ValueError(f"qk_norm_rope_store: cache shape {tuple(k_cache.shape)}")
        if k_cache.stride() != v_cache.stride():
            raise ValueError("qk_norm_rope_store: k_cache and v_cache strides differ")
        if block_mapping.shape != (T,) or slot_mapping.shape != (T,):
            raise ValueError(f"qk_norm_rope_store: mappings must have shape ({T},)")
        itag = index_tag(block_mapping, "block_mapping")
        bm = block_mapping.contiguous()
        sm = slot_mapping.to(bm.dtype).contiguous()
        keep += [bm, sm]
        a.v = v.data_ptr()
        a.v_stride_token, a.v_stride_head = _heads_view(v, "v")
        a.k_cache, a.v_cache = k_cache.data_ptr(), v_cache.data_ptr()
        for i, s in enumerate(k_cache.stride()):
            a.cache_strides[i] = s
        a.num_blocks, a.block_size = k_cache.shape[0], k_cache.shape[2]
        a.block_mapping, a.slot_mapping, a.index_type = bm.data_ptr(), sm.data_ptr(), itag
    a.num_tokens, a.num_q_heads, a.num_kv_heads, a.head_dim = T, Hq, Hkv, D
    a.dtype = tag
    a.status = status_word(dev).data_ptr()
    with on_device(dev):
        rc = _capi.lib().qf_qk_norm_rope_store(ctypes.byref(a), stream_ptr(dev))
    _capi.check(rc, "qk_norm_rope_store")
    after_op(dev)
    return q_out, k_out


def apply_rotary_pos_emb(q: torch.Tensor, k: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                         unsqueeze_dim: int = 1) -> tuple[torch.Tensor, torch.Tensor]:
    """Drop-in for transformers' ``apply_rotary_pos_emb`` (modeling_qwen3.py:159).

    q: (B, Hq, T, D) with unsqueeze_dim=1, or (B, T, Hq, D) with unsqueeze_dim=2;
    cos/sin: (B, T, D).  Returns new tensors of q's and k's shapes whose memory
    is token-major (what the attention kernels read)."""
    if q.dim() != 4 or k.dim() != 4 or unsqueeze_dim not in (1, 2):
        raise ValueError("apply_rotary_pos_emb: q/k must be 4D, unsqueeze_dim 1 or 2")
    if cos.dim() == 2:
        cos, sin = cos.unsqueeze(0), sin.unsqueeze(0)
    qs, ks = [], []
    for b in range(q.shape[0]):
        qb, kb = q[b], k[b]
        if unsqueeze_dim == 1:  # (H, T, D) -> (T, H, D) view
            qb, kb = qb.transpose(0, 1), kb.transpose(0, 1)
        cb = cos[b if cos.shape[0] > 1 else 0]
        sb = sin[b if sin.shape[0] > 1 else 0]
        qo, ko = qk_norm_rope_store(qb, kb, None, None, None, 0.0, cb, sb)
        if unsqueeze_dim == 1:
            qo, ko = qo.transpose(0, 1), ko.transpose(0, 1)
        qs.append(qo)
        ks.append(ko)
    return torch.stack(qs) if len(qs) > 1 else qs[0].unsqueeze(0), \
        torch.stack(ks) if len(ks) > 1 else ks[0].unsqueeze(0)


# ----------------------------------------------------------------------------
def silu_and_mul(gate: torch.Tensor, up: torch.Tensor | None = None,
                 out: torch.Tensor | None = None) -> torch.Tensor:
    """``silu(gate) * up``.  With ``up=None``, ``gate`` is the merged [..., 2I]
    gate|up projection (gate first)."""
    if up is None:
        I2 = gate.shape[-1]
        if I2 % 2:
            raise ValueError("silu_and_mul: merged input needs an even last dim")
        g2 = _rows(gate)
        I = I2 // 2
        g_rows, u_rows = g2[:, :I], g2[:, I:]
        out_shape = (*gate.shape[:-1], I)
    else:
        if gate.shape != up.shape:
            raise ValueError(f"silu_and_mul: gate {tuple(gate.shape)} vs up {tuple(up.shape)}")
        g_rows, u_rows = _rows(gate), _rows(up)
        I = gate.shape[-1]
        out_shape = tuple(gate.shape)
    if g_rows.dtype != u_rows.dtype:
        raise ValueError("silu_and_mul: gate and up dtypes differ")
    tag = dtype_tag(g_rows, "silu_and_mul")
    dev = require_cuda("silu_and_mul", g_rows, u_rows, out)
    if out is None:
        out = torch.empty(out_shape, dtype=g_rows.dtype, device=dev)
    o2 = out.view(-1, I)
    with on_device(dev):
        rc = _capi.lib().qf_silu_and_mul(g_rows.data_ptr(), g_rows.stride(0), u_rows.data_ptr(),
                                         u_rows.stride(0), o2.data_ptr(), o2.stride(0),
                                         g_rows.shape[0], I, tag, stream_ptr(dev))
    _capi.check(rc, "silu_and_mul")
    return out


# ----------------------------------------------------------------------------
def build_slot_mapping(cu_seqlens: torch.Tensor, positions: torch.Tensor,
                       block_tables: torch.Tensor, block_size: int
                       ) -> tuple[torch.Tensor, torch.Tensor]:
    """(block_mapping, slot_mapping), int64 (T,), for tokens grouped into
    sequences by ``cu_seqlens`` (S+1,) int32 at absolute ``positions`` (T,)
    int64, with ``block_tables`` (S, max_blocks) int32."""
    dev = require_cuda("build_slot_mapping", cu_seqlens, positions, block_tables)
    cu = cu_seqlens.to(torch.int32).contiguous()
    pos = positions.reshape(-1).to(torch.int64).contiguous()
    bt = block_tables.to(torch.int32)
    if bt.dim() != 2 or bt.stride(1) != 1:
        bt = bt.contiguous()
    T = pos.numel()
    bm = torch.empty(T, dtype=torch.int64, device=dev)
    sm = torch.empty(T, dtype=torch.int64, device=dev)
    with on_device(dev):
        rc = _capi.lib().qf_build_slot_mapping(cu.data_ptr(), cu.numel() - 1, pos.data_ptr(), T,
                                               bt.data_ptr(), bt.stride(0), bt.shape[1],
                                               int(block_size), bm.data_ptr(), sm.data_ptr(),
                                               status_word(dev).data_ptr(), stream_ptr(dev))
    _capi.check(rc, "build_slot_mapping")
    after_op(dev)
    return bm, sm
