"""Paged KV-cache store with the reference's operator signatures.

Drop-in for ``server/model/kernels/kv_cache.py`` of tinyserver: same function
names, arguments, in-place semantics and ``ValueError`` contract (validation
happens before any device work, so the reference's CPU-only validation tests
hold).  The work runs in libqwen3fused's sm_100a store kernel
(``qf_kv_store_seq`` / ``qf_kv_store_batched``) on the current CUDA stream.

Differences a caller can observe:

* a block/slot outside the cache is never written (the reference's Triton
  kernel would write out of bounds); it is reported through
  :func:`tinyserver_b200.check_errors`;
* ``store_kv_cache`` also requires ``v_src.shape == k_src.shape`` (the
  reference reads V with K's shape and strides).
"""

from __future__ import annotations

import torch

from .. import _capi
from .._runtime import after_op, index_tag, on_device, require_cuda, status_word, stream_ptr

__all__ = ["store_kv_cache", "store_kv_cache_batched"]


def _check_caches(k_cache: torch.Tensor, v_cache: torch.Tensor, k_src: torch.Tensor) -> None:
    if k_cache.dim() != 4 or v_cache.dim() != 4:
        raise ValueError(
            f"k_cache and v_cache must be 4D tensors (num_blocks, num_kv_heads, block_size, "
            f"head_dim), but got shapes {k_cache.shape} and {v_cache.shape}")
    if k_cache.shape != v_cache.shape:
        raise ValueError(f"k_cache and v_cache must have the same shape, but got "
                         f"{k_cache.shape} and {v_cache.shape}")
    num_kv_heads, _, head_dim = k_src.shape
    if k_cache.shape[1] != num_kv_heads or k_cache.shape[3] != head_dim:
        raise ValueError(f"cache shape {tuple(k_cache.shape)} does not match k_src "
                         f"(num_kv_heads={num_kv_heads}, head_dim={head_dim})")
    if not (k_src.dtype == k_cache.dtype == v_cache.dtype):
        raise ValueError(f"k_src/v_src/k_cache/v_cache dtypes differ: {k_src.dtype}, "
                         f"{k_cache.dtype}, {v_cache.dtype}")


def store_kv_cache(
    start_position: int,
    block_table: torch.Tensor,
    k_src: torch.Tensor,
    v_src: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
) -> None:
    """Scatter one sequence's K/V rows into the paged cache.

    Same contract as the reference's ``store_kv_cache`` (kv_cache.py:73-119):
    token i of ``k_src``/``v_src`` (num_kv_heads, seq_len, head_dim) is at
    absolute position ``start_position + i`` and lands in block
    ``block_table[pos // block_size]``, slot ``pos % block_size``.
    """
    if k_src.dim() != 3 or v_src.dim() != 3:
        raise ValueError(
            f"k_src and v_src must be 3D tensors, but got shapes {k_src.shape} and {v_src.shape}"
        )
    if k_src.shape != v_src.shape:
        raise ValueError(
            f"k_src and v_src must have the same shape, but got {k_src.shape} and {v_src.shape}"
        )
    if v_src.dtype != k_src.dtype:
        raise ValueError(f"k_src and v_src dtypes differ: {k_src.dtype} and {v_src.dtype}")
    _check_caches(k_cache, v_cache, k_src)
    start_position = int(start_position)
    if start_position < 0:
        raise ValueError(f"start_position must be >= 0, got {start_position}")
    if block_table.dim() != 1:
        raise ValueError(f"block_table must be 1D, got shape {block_table.shape}")
    itag = index_tag(block_table, "store_kv_cache block_table")
    dev = require_cuda("store_kv_cache", block_table, k_src, v_src, k_cache, v_cache)
    num_kv_heads, num_tokens, head_dim = k_src.shape
    if block_table.stride(0) != 1 and block_table.numel() > 1:
        block_table = block_table.contiguous()
    with on_device(dev):
        rc = _capi.lib().qf_kv_store_seq(
            start_position, block_table.data_ptr(), block_table.numel(), itag,
            k_src.data_ptr(), _capi.i64_array(k_src.stride()),
            v_src.data_ptr(), _capi.i64_array(v_src.stride()),
            k_cache.data_ptr(), _capi.i64_array(k_cache.stride()),
            v_cache.data_ptr(), _capi.i64_array(v_cache.stride()),
            num_tokens, num_kv_heads, head_dim, k_cache.shape[0], k_cache.shape[2],
            k_src.element_size(), status_word(dev).data_ptr(), stream_ptr(dev))
    _capi.check(rc, "store_kv_cache")
    after_op(dev)


def store_kv_cache_batched(
    k_src: torch.Tensor,
    v_src: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    block_mapping: torch.Tensor,
    slot_mapping: torch.Tensor,
) -> None:
    """Scatter a whole batch's K/V rows: ``cache[block_mapping[t], h, slot_mapping[t]]
    = src[h, t]``.

    Same contract as the reference's ``store_kv_cache_batched``
    (kv_cache.py:194-251); the mappings may be int32 or int64.
    """
    if k_src.dim() != 3 or v_src.dim() != 3:
        raise ValueError(
            f"k_src and v_src must be 3D tensors, but got shapes {k_src.shape} and {v_src.shape}"
        )
    if k_src.shape != v_src.shape:
        raise ValueError(
            f"k_src and v_src must have the same shape, but got {k_src.shape} and {v_src.shape}"
        )

    num_key_value_heads, num_tokens, head_dim = k_src.shape

    if block_mapping.shape[0] != num_tokens or slot_mapping.shape[0] != num_tokens:
        raise ValueError(
            f"block_mapping and slot_mapping must have length num_tokens ({num_tokens}), "
            f"but got {block_mapping.shape[0]} and {slot_mapping.shape[0]}"
        )
    if v_src.dtype != k_src.dtype:
        raise ValueError(f"k_src and v_src dtypes differ: {k_src.dtype} and {v_src.dtype}")
    _check_caches(k_cache, v_cache, k_src)
    if block_mapping.dim() != 1 or slot_mapping.dim() != 1:
        raise ValueError("block_mapping and slot_mapping must be 1D")
    itag = index_tag(block_mapping, "store_kv_cache_batched block_mapping")
    if slot_mapping.dtype != block_mapping.dtype:
        slot_mapping = slot_mapping.to(block_mapping.dtype)
    dev = require_cuda("store_kv_cache_batched", k_src, v_src, k_cache, v_cache, block_mapping,
                       slot_mapping)
    block_mapping = block_mapping.contiguous()
    slot_mapping = slot_mapping.contiguous()
    with on_device(dev):
        rc = _capi.lib().qf_kv_store_batched(
            k_src.data_ptr(), _capi.i64_array(k_src.stride()),
            v_src.data_ptr(), _capi.i64_array(v_src.stride()),
            k_cache.data_ptr(), _capi.i64_array(k_cache.stride()),
            v_cache.data_ptr(), _capi.i64_array(v_cache.stride()),
            block_mapping.data_ptr(), slot_mapping.data_ptr(), itag,
            num_tokens, num_key_value_heads, head_dim, k_cache.shape[0], k_cache.shape[2],
            k_src.element_size(), status_word(dev).data_ptr(), stream_ptr(dev))
    _capi.check(rc, "store_kv_cache_batched")
    after_op(dev)
