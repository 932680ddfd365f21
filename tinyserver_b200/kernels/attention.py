"""Attention on B200 (CUDA only, no fallback): decode paged attention over
the (num_blocks, num_kv_heads, block_size, head_dim) KV pages the fused store
writes, and prefill attention over packed variable-length sequences.

:func:`paged_attention_forward` has the signature and contract of the
reference's ``paged_attention_forward`` (server/model/kernels/
paged_attention.py:124-192): one query token per sequence, GQA heads grouped
contiguously, softmax scale 1/sqrt(head_dim), fp32 math, output in the
query's dtype.
"""

from __future__ import annotations

import math

import torch

from .. import _capi
from .._runtime import (after_op, dtype_tag, on_device, require_cuda, status_word, stream_ptr,
                        work_counter)

__all__ = ["flash_attn_varlen_func", "paged_attention_forward", "paged_attention_workspace_bytes"]


def paged_attention_workspace_bytes(num_seqs: int, num_q_heads: int, head_dim: int,
                                    max_seq_len: int) -> int:
    """Bytes of fp32 scratch that let sequences of up to ``max_seq_len`` tokens
    be split over several CTAs (0 when nothing needs splitting)."""
    return int(_capi.lib().qf_paged_attention_workspace_bytes(num_seqs, num_q_heads, head_dim,
                                                              max_seq_len))


def paged_attention_forward(query: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                            block_tables: torch.Tensor, block_size: int,
                            seq_lens: torch.Tensor, *, workspace: torch.Tensor | None = None,
                            split: bool = True) -> torch.Tensor:
    """out[s, h] = softmax(query[s, h] @ K_s.T / sqrt(D)) @ V_s over the first
    ``seq_lens[s]`` cached tokens of sequence s (block_tables[s] maps its
    logical blocks to cache blocks).  Returns a new tensor shaped like query.

    ``split`` lets long sequences spread over several CTAs through an fp32
    workspace (allocated here unless ``workspace`` is given)."""
    if query.dim() != 3:
        raise ValueError(f"query must be a 3D tensor, but got shape {query.shape}")
    if k_cache.dim() != 4 or v_cache.shape != k_cache.shape:
        raise ValueError("k_cache/v_cache must be (num_blocks, num_kv_heads, block_size, "
                         f"head_dim), got {tuple(k_cache.shape)} and {tuple(v_cache.shape)}")
    if k_cache.stride() != v_cache.stride():
        raise ValueError("k_cache and v_cache strides differ")
    S, Hq, D = query.shape
    N, Hkv, B, Dc = k_cache.shape
    if Dc != D or B != block_size:
        raise ValueError(f"cache geometry {tuple(k_cache.shape)} does not match head_dim {D} "
                         f"/ block_size {block_size}")
    if Hq % Hkv:
        raise ValueError(f"num_heads {Hq} is not a multiple of num_kv_heads {Hkv}")
    if block_tables.dim() != 2 or block_tables.shape[0] != S or seq_lens.shape != (S,):
        raise ValueError("block_tables must be (num_seqs, max_blocks) and seq_lens (num_seqs,)")
    if query.dtype != k_cache.dtype:
        raise ValueError(f"query dtype {query.dtype} != cache dtype {k_cache.dtype}")
    tag = dtype_tag(query, "paged_attention_forward")
    dev = require_cuda("paged_attention_forward", query, k_cache, v_cache, block_tables,
                       seq_lens, workspace)
    q = query if query.stride(2) == 1 else query.contiguous()
    bt = block_tables.to(torch.int32)
    if bt.stride(1) != 1:
        bt = bt.contiguous()
    lens = seq_lens.to(torch.int32).contiguous()
    out = torch.empty_like(q)
    a = _capi.PagedAttentionArgs()
    a.q, a.q_stride_seq, a.q_stride_head = q.data_ptr(), q.stride(0), q.stride(1)
    a.k_cache, a.v_cache = k_cache.data_ptr(), v_cache.data_ptr()
    for i in range(4):
        a.cache_strides[i] = k_cache.stride(i)
    a.num_blocks, a.block_size = N, B
    a.block_tables, a.block_tables_row_stride = bt.data_ptr(), bt.stride(0)
    a.max_blocks_per_seq = bt.shape[1]
    a.seq_lens = lens.data_ptr()
    a.num_seqs, a.num_q_heads, a.num_kv_heads, a.head_dim = S, Hq, Hkv, D
    a.scale = 1.0 / math.sqrt(D)
    a.out, a.out_stride_seq, a.out_stride_head = out.data_ptr(), out.stride(0), out.stride(1)
    if split:
        need = paged_attention_workspace_bytes(S, Hq, D, max(1, bt.shape[1] * B))
        if need and workspace is None:
            workspace = torch.empty(need // 4, dtype=torch.float32, device=dev)
        if workspace is not None:
            a.workspace, a.workspace_bytes = workspace.data_ptr(), \
                workspace.numel() * workspace.element_size()
    a.dtype = tag
    a.status = status_word(dev).data_ptr()
    with on_device(dev):
        rc = _capi.lib().qf_paged_attention_decode(a, stream_ptr(dev))
    _capi.check(rc, "paged_attention_forward")
    after_op(dev)
    return out


def flash_attn_varlen_func(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                           cu_seqlens_q: torch.Tensor, cu_seqlens_k: torch.Tensor,
                           max_seqlen_q: int, max_seqlen_k: int, causal: bool,
                           softmax_scale: float | None = None) -> torch.Tensor:
    """Prefill attention over packed variable-length sequences, with the
    signature and contract of the reference's ``flash_attn_varlen_func``
    (server/model/kernels/varlen_attention.py:145-218): q (Tq, Hq, D), k/v
    (Tk, Hkv, D), sequence b at rows [cu_seqlens[b], cu_seqlens[b+1]), GQA
    heads grouped contiguously, causal masking within each sequence, scale
    1/sqrt(D) unless given.  Returns a new tensor shaped like q."""
    if q.dim() != 3 or k.dim() != 3 or v.dim() != 3:
        raise ValueError("q, k, v must be 3D tensors")
    Tq, Hq, D = q.shape
    Tk, Hkv, Dk = k.shape
    if Hq % Hkv != 0:
        raise ValueError("num_heads_q must be divisible by num_heads_k for GQA")
    if v.shape != k.shape or Dk != D:
        raise ValueError(f"k {tuple(k.shape)} / v {tuple(v.shape)} do not match q {tuple(q.shape)}")
    if not (q.dtype == k.dtype == v.dtype):
        raise ValueError("q, k and v must share a dtype")
    if cu_seqlens_q.shape != cu_seqlens_k.shape or cu_seqlens_q.dim() != 1:
        raise ValueError("cu_seqlens_q and cu_seqlens_k must be (batch + 1,)")
    tag = dtype_tag(q, "flash_attn_varlen_func")
    dev = require_cuda("flash_attn_varlen_func", q, k, v, cu_seqlens_q, cu_seqlens_k)
    qq, kk, vv = (t if t.stride(2) == 1 else t.contiguous() for t in (q, k, v))
    cq = cu_seqlens_q.to(torch.int32).contiguous()
    ck = cu_seqlens_k.to(torch.int32).contiguous()
    out = torch.empty_like(qq)
    a = _capi.VarlenAttentionArgs()
    a.q, a.q_stride_token, a.q_stride_head = qq.data_ptr(), qq.stride(0), qq.stride(1)
    a.k, a.k_stride_token, a.k_stride_head = kk.data_ptr(), kk.stride(0), kk.stride(1)
    a.v, a.v_stride_token, a.v_stride_head = vv.data_ptr(), vv.stride(0), vv.stride(1)
    a.out, a.out_stride_token, a.out_stride_head = out.data_ptr(), out.stride(0), out.stride(1)
    a.cu_seqlens_q, a.cu_seqlens_k = cq.data_ptr(), ck.data_ptr()
    a.batch, a.max_seqlen_q = cq.numel() - 1, int(max_seqlen_q)
    a.num_q_heads, a.num_kv_heads, a.head_dim = Hq, Hkv, D
    a.causal = 1 if causal else 0
    a.scale = float(softmax_scale) if softmax_scale is not None else 1.0 / math.sqrt(D)
    a.dtype = tag
    a.status = status_word(dev).data_ptr()
    a.total_q, a.total_k = Tq, Tk
    a.work_counter = work_counter(dev).data_ptr()
    with on_device(dev):
        rc = _capi.lib().qf_varlen_attention(a, stream_ptr(dev))
    _capi.check(rc, "flash_attn_varlen_func")
    after_op(dev)
    return out
