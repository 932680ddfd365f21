"""ctypes binding of libqwen3fused.so (declared in include/qwen3fused.h).

The library is built in-tree (``python -m tinyserver_b200.build``).  If it is
missing or older than its sources it is rebuilt once per process; if that
fails, every op raises -- there is no CPU or torch fallback.
"""

from __future__ import annotations

import ctypes
import os
import threading

from . import build as _build

c_i64 = ctypes.c_int64
c_int = ctypes.c_int
c_vp = ctypes.c_void_p
c_float = ctypes.c_float
I64P = ctypes.POINTER(ctypes.c_int64)

QF_F32, QF_F16, QF_BF16 = 0, 1, 2
QF_I32, QF_I64 = 0, 1
QF_OK, QF_ERR_INVALID, QF_ERR_UNSUPPORTED, QF_ERR_LAUNCH, QF_ERR_DEVICE = 0, 1, 2, 3, 4
QF_ERR_SCRATCH = 5
QF_FLAG_BAD_BLOCK, QF_FLAG_BAD_SLOT, QF_FLAG_BAD_TOKEN, QF_FLAG_BAD_TABLE = 1, 2, 4, 8
QF_FLAG_TIMEOUT = 16

FLAG_NAMES = {QF_FLAG_BAD_BLOCK: "block index outside the cache",
              QF_FLAG_BAD_SLOT: "slot index outside the block",
              QF_FLAG_BAD_TOKEN: "token id outside the vocabulary",
              QF_FLAG_BAD_TABLE: "position beyond the block table",
              QF_FLAG_TIMEOUT: "a kernel timed out waiting on its tensor-core work"}


class QkNormRopeArgs(ctypes.Structure):
    """Mirror of qf_qk_norm_rope_args (field order and types must match)."""

    _fields_ = [
        ("q", c_vp), ("q_stride_token", c_i64), ("q_stride_head", c_i64),
        ("k", c_vp), ("k_stride_token", c_i64), ("k_stride_head", c_i64),
        ("v", c_vp), ("v_stride_token", c_i64), ("v_stride_head", c_i64),
        ("q_weight", c_vp), ("k_weight", c_vp), ("eps", c_float),
        ("cos", c_vp), ("sin", c_vp), ("cos_sin_token_stride", c_i64),
        ("positions", c_vp), ("positions_type", c_int), ("inv_freq", c_vp),
        ("q_out", c_vp), ("q_out_stride_token", c_i64), ("q_out_stride_head", c_i64),
        ("k_out", c_vp), ("k_out_stride_token", c_i64), ("k_out_stride_head", c_i64),
        ("k_cache", c_vp), ("v_cache", c_vp), ("cache_strides", c_i64 * 4),
        ("num_blocks", c_i64), ("block_size", c_i64),
        ("block_mapping", c_vp), ("slot_mapping", c_vp), ("index_type", c_int),
        ("num_tokens", c_i64), ("num_q_heads", c_i64), ("num_kv_heads", c_i64),
        ("head_dim", c_i64),
        ("dtype", c_int),
        ("status", c_vp),
    ]


class PagedAttentionArgs(ctypes.Structure):
    """Mirror of qf_paged_attention_args (field order and types must match)."""

    _fields_ = [
        ("q", c_vp), ("q_stride_seq", c_i64), ("q_stride_head", c_i64),
        ("k_cache", c_vp), ("v_cache", c_vp), ("cache_strides", c_i64 * 4),
        ("num_blocks", c_i64), ("block_size", c_i64),
        ("block_tables", c_vp), ("block_tables_row_stride", c_i64),
        ("max_blocks_per_seq", c_i64),
        ("seq_lens", c_vp),
        ("num_seqs", c_i64), ("num_q_heads", c_i64), ("num_kv_heads", c_i64),
        ("head_dim", c_i64),
        ("scale", c_float),
        ("out", c_vp), ("out_stride_seq", c_i64), ("out_stride_head", c_i64),
        ("workspace", c_vp), ("workspace_bytes", c_i64),
        ("dtype", c_int),
        ("status", c_vp),
    ]


class VarlenAttentionArgs(ctypes.Structure):
    """Mirror of qf_varlen_attention_args (field order and types must match)."""

    _fields_ = [
        ("q", c_vp), ("q_stride_token", c_i64), ("q_stride_head", c_i64),
        ("k", c_vp), ("k_stride_token", c_i64), ("k_stride_head", c_i64),
        ("v", c_vp), ("v_stride_token", c_i64), ("v_stride_head", c_i64),
        ("out", c_vp), ("out_stride_token", c_i64), ("out_stride_head", c_i64),
        ("cu_seqlens_q", c_vp), ("cu_seqlens_k", c_vp),
        ("batch", c_i64), ("max_seqlen_q", c_i64), ("num_q_heads", c_i64),
        ("num_kv_heads", c_i64), ("head_dim", c_i64),
        ("causal", c_int),
        ("scale", c_float),
        ("dtype", c_int),
        ("status", c_vp),
        ("total_q", c_i64), ("total_k", c_i64),
        ("work_counter", c_vp),
    ]


class SampleArgs(ctypes.Structure):
    """Mirror of qf_sample_args (field order and types must match)."""

    _fields_ = [
        ("logits", c_vp), ("logits_row_stride", c_i64),
        ("batch", c_i64), ("vocab", c_i64),
        ("dtype", c_int),
        ("temperature", c_vp),
        ("top_k", c_vp), ("top_k_type", c_int),
        ("top_p", c_vp),
        ("uniforms", c_vp),
        ("seeds", c_vp), ("steps", c_vp),
        ("out", c_vp),
        ("workspace", c_vp), ("workspace_bytes", c_i64),
        ("path", c_int),
    ]


# name -> argtypes of every exported entry point (restype int unless listed below)
SIGNATURES: dict[str, list] = {
    "qf_kv_store_batched": [c_vp, I64P, c_vp, I64P, c_vp, I64P, c_vp, I64P, c_vp, c_vp, c_int,
                            c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_vp, c_vp],
    "qf_kv_store_seq": [c_i64, c_vp, c_i64, c_int, c_vp, I64P, c_vp, I64P, c_vp, I64P, c_vp,
                        I64P, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_vp, c_vp],
    "qf_rmsnorm": [c_vp, c_i64, c_vp, c_vp, c_i64, c_i64, c_i64, c_float, c_int, c_vp],
    "qf_add_rmsnorm": [c_vp, c_i64, c_vp, c_i64, c_vp, c_vp, c_i64, c_vp, c_i64, c_i64, c_i64,
                       c_float, c_int, c_vp],
    "qf_rope_cos_sin": [c_vp, c_int, c_vp, c_i64, c_i64, c_float, c_int, c_vp, c_vp, c_vp],
    "qf_qk_norm_rope_store": [ctypes.POINTER(QkNormRopeArgs), c_vp],
    "qf_qk_norm_rope_args_size": [],
    "qf_silu_and_mul": [c_vp, c_i64, c_vp, c_i64, c_vp, c_i64, c_i64, c_i64, c_int, c_vp],
    "qf_embedding": [c_vp, c_int, c_vp, c_i64, c_i64, c_vp, c_i64, c_i64, c_i64, c_i64, c_vp,
                     c_vp],
    "qf_build_slot_mapping": [c_vp, c_i64, c_vp, c_i64, c_vp, c_i64, c_i64, c_i64, c_vp, c_vp,
                              c_vp, c_vp],
    "qf_paged_attention_decode": [ctypes.POINTER(PagedAttentionArgs), c_vp],
    "qf_paged_attention_workspace_bytes": [c_i64, c_i64, c_i64, c_i64],
    "qf_paged_attention_args_size": [],
    "qf_paged_attention_decode_noalloc": [ctypes.POINTER(PagedAttentionArgs), c_vp],
    "qf_paged_attention_noalloc_capacity": [],
    "qf_varlen_attention": [ctypes.POINTER(VarlenAttentionArgs), c_vp],
    "qf_varlen_attention_args_size": [],
    "qf_sample_tokens": [ctypes.POINTER(SampleArgs), c_vp],
    "qf_sample_workspace_bytes": [c_i64],
    "qf_sample_args_size": [],
    "qf_uniforms_from_seeds": [c_vp, c_vp, c_i64, c_vp, c_vp],
    "qf_read_status": [c_vp, ctypes.POINTER(ctypes.c_int32), c_int, c_vp],
    "qf_last_cuda_error": [],
    "qf_version": [],
}
RESTYPES = {"qf_last_cuda_error": ctypes.c_char_p, "qf_version": ctypes.c_char_p,
            "qf_qk_norm_rope_args_size": ctypes.c_size_t,
            "qf_paged_attention_args_size": ctypes.c_size_t,
            "qf_paged_attention_workspace_bytes": ctypes.c_size_t,
            "qf_paged_attention_noalloc_capacity": ctypes.c_size_t,
            "qf_sample_workspace_bytes": c_i64,
            "qf_varlen_attention_args_size": ctypes.c_size_t,
            "qf_sample_args_size": ctypes.c_size_t}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def ensure_built() -> str:
    """Return the library path, (re)building it when its sources changed (the
    sources' hash decides; concurrent processes take turns, see build.build)."""
    if _build.is_stale():
        _build.build()
    return _build.LIB


def lib() -> ctypes.CDLL:
    """Load libqwen3fused.so once (building it first if needed)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            path = ensure_built()
            handle = ctypes.CDLL(path)
            for name, argtypes in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.argtypes = argtypes
                fn.restype = RESTYPES.get(name, c_int)
            for fn, mirror in (("qf_qk_norm_rope_args_size", QkNormRopeArgs),
                               ("qf_paged_attention_args_size", PagedAttentionArgs),
                               ("qf_varlen_attention_args_size", VarlenAttentionArgs),
                               ("qf_sample_args_size", SampleArgs)):
                size = getattr(handle, fn)()
                if size != ctypes.sizeof(mirror):
                    raise RuntimeError(f"{fn}: ABI mismatch, library {size} bytes, binding "
                                       f"{ctypes.sizeof(mirror)} bytes")
            _lib = handle
    return _lib


def lib_path() -> str:
    return _build.LIB


def check(rc: int, what: str) -> None:
    """Turn a QF_* return code into the exception the reference would raise."""
    if rc == QF_OK:
        return
    if rc == QF_ERR_INVALID:
        raise ValueError(f"{what}: invalid argument")
    if rc == QF_ERR_UNSUPPORTED:
        raise ValueError(f"{what}: unsupported shape, stride or alignment")
    if rc == QF_ERR_LAUNCH:
        err = lib().qf_last_cuda_error().decode()
        raise RuntimeError(f"{what}: CUDA launch failed: {err}")
    raise RuntimeError(f"{what}: error code {rc}")


def i64_array(vals) -> ctypes.Array:
    return (c_i64 * len(vals))(*[int(v) for v in vals])
