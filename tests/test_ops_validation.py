"""Host-side contract of the reference-compatible operators (CPU only).

The first three tests are the reference's own CPU validation cases
(tests/model/test_kv_cache_kernels.py:210-255) pointed at the drop-in: the
same ValueErrors, raised before any device work.  The rest check that the
library has no CPU path: CPU tensors are rejected, never computed.
"""

import pytest
import torch

import tinyserver_b200 as tsb
from tinyserver_b200.kernels.kv_cache import store_kv_cache, store_kv_cache_batched


def test_batched_wrong_k_src_dim_raises():
    num_kv_heads, head_dim = 2, 8
    k_src = torch.zeros(num_kv_heads, head_dim)
    v_src = torch.zeros(num_kv_heads, 1, head_dim)
    k_cache = torch.zeros(1, num_kv_heads, 4, head_dim)
    v_cache = torch.zeros_like(k_cache)
    bm = torch.zeros(1, dtype=torch.int32)
    sm = torch.zeros(1, dtype=torch.int32)
    with pytest.raises(ValueError, match="3D"):
        store_kv_cache_batched(k_src, v_src, k_cache, v_cache, bm, sm)


def test_batched_kv_shape_mismatch_raises():
    k_src = torch.zeros(2, 3, 8)
    v_src = torch.zeros(2, 4, 8)
    k_cache = torch.zeros(2, 2, 4, 8)
    with pytest.raises(ValueError):
        store_kv_cache_batched(k_src, v_src, k_cache, torch.zeros_like(k_cache),
                               torch.zeros(3, dtype=torch.int32), torch.zeros(3, dtype=torch.int32))


def test_batched_block_mapping_length_mismatch_raises():
    k_src = torch.zeros(2, 4, 8)
    k_cache = torch.zeros(2, 2, 4, 8)
    with pytest.raises(ValueError):
        store_kv_cache_batched(k_src, torch.zeros_like(k_src), k_cache, torch.zeros_like(k_cache),
                               torch.zeros(3, dtype=torch.int32), torch.zeros(4, dtype=torch.int32))


def test_per_seq_wrong_dim_raises():
    with pytest.raises(ValueError, match="3D"):
        store_kv_cache(0, torch.zeros(1, dtype=torch.int32), torch.zeros(2, 8),
                       torch.zeros(2, 1, 8), torch.zeros(1, 2, 4, 8), torch.zeros(1, 2, 4, 8))


def test_cache_geometry_mismatch_raises():
    with pytest.raises(ValueError, match="does not match"):
        store_kv_cache_batched(torch.zeros(2, 1, 8), torch.zeros(2, 1, 8),
                               torch.zeros(1, 3, 4, 8), torch.zeros(1, 3, 4, 8),
                               torch.zeros(1, dtype=torch.long), torch.zeros(1, dtype=torch.long))


def test_cpu_tensors_are_rejected_not_computed():
    k = torch.zeros(2, 1, 8)
    kc = torch.zeros(1, 2, 4, 8)
    with pytest.raises(ValueError, match="CUDA tensors only"):
        store_kv_cache_batched(k, k, kc, kc.clone(), torch.zeros(1, dtype=torch.long),
                               torch.zeros(1, dtype=torch.long))
    with pytest.raises(ValueError, match="CUDA tensors only"):
        store_kv_cache(0, torch.zeros(1, dtype=torch.int32), k, k, kc, kc.clone())
    x = torch.zeros(3, 16)
    w = torch.ones(16)
    with pytest.raises(ValueError, match="CUDA tensors only"):
        tsb.rms_norm(x, w, 1e-6)
    with pytest.raises(ValueError, match="CUDA tensors only"):
        tsb.fused_add_rms_norm(x, x, w, 1e-6)
    with pytest.raises(ValueError, match="CUDA tensors only"):
        tsb.silu_and_mul(torch.zeros(3, 32))
    with pytest.raises(ValueError, match="CUDA tensors only"):
        tsb.embedding(torch.zeros(3, dtype=torch.long), torch.zeros(10, 16))
    with pytest.raises(ValueError, match="CUDA tensors only"):
        tsb.qk_norm_rope_store(torch.zeros(2, 2, 128), torch.zeros(2, 1, 128), None, None, None,
                               1e-6, torch.zeros(2, 128), torch.zeros(2, 128))
    with pytest.raises(ValueError, match="CUDA tensors only"):
        tsb.rope_cos_sin(torch.zeros(3, dtype=torch.long), torch.zeros(64), 128, torch.bfloat16)


def test_unsupported_dtypes_raise():
    with pytest.raises(ValueError, match="index dtype"):
        store_kv_cache_batched(torch.zeros(2, 1, 8), torch.zeros(2, 1, 8), torch.zeros(1, 2, 4, 8),
                               torch.zeros(1, 2, 4, 8), torch.zeros(1, dtype=torch.float32),
                               torch.zeros(1, dtype=torch.float32))
    with pytest.raises(ValueError, match="dtype"):
        tsb.rms_norm(torch.zeros(2, 8, dtype=torch.float64), torch.ones(8, dtype=torch.float64),
                     1e-6)


def test_paged_attention_rejects_a_2d_query():
    """Same guard as the reference (paged_attention.py:171-172), before any device work."""
    from tinyserver_b200 import paged_attention_forward

    query = torch.zeros(4, 64)
    k_cache = torch.zeros(2, 4, 16, 64)
    with pytest.raises(ValueError, match="3D"):
        paged_attention_forward(query, k_cache, torch.zeros_like(k_cache),
                                torch.zeros(1, 1, dtype=torch.int32), 16,
                                torch.ones(1, dtype=torch.int32))


def test_paged_attention_rejects_cpu_tensors():
    from tinyserver_b200 import paged_attention_forward

    k_cache = torch.zeros(2, 4, 16, 64)
    with pytest.raises(ValueError, match="CUDA tensors only"):
        paged_attention_forward(torch.zeros(1, 4, 64), k_cache, torch.zeros_like(k_cache),
                                torch.zeros(1, 1, dtype=torch.int32), 16,
                                torch.ones(1, dtype=torch.int32))


def test_varlen_attention_rejects_a_2d_input():
    """Same guard as the reference (varlen_attention.py:171-172)."""
    from tinyserver_b200 import flash_attn_varlen_func

    cu = torch.tensor([0, 4], dtype=torch.int32)
    with pytest.raises(ValueError, match="3D"):
        flash_attn_varlen_func(torch.zeros(4, 64), torch.zeros(4, 1, 64), torch.zeros(4, 1, 64),
                               cu, cu, 4, 4, True)
    with pytest.raises(ValueError, match="divisible"):
        flash_attn_varlen_func(torch.zeros(4, 3, 64), torch.zeros(4, 2, 64),
                               torch.zeros(4, 2, 64), cu, cu, 4, 4, True)


def test_sample_tokens_rejects_bad_shapes_like_the_reference():
    """The reference's shape errors (tests/model/test_batch_sampling.py
    test_rejects_bad_shapes): same messages, raised before any device work."""
    with pytest.raises(ValueError, match="Expected logits shape"):
        tsb.sample_tokens(torch.randn(10), torch.ones(1), torch.zeros(1, dtype=torch.int64),
                          torch.ones(1), torch.ones(1) * 0.5)
    with pytest.raises(ValueError, match="Expected top_k shape"):
        tsb.sample_tokens(torch.randn(2, 10), torch.ones(2), torch.zeros(3, dtype=torch.int64),
                          torch.ones(2), torch.ones(2) * 0.5)
    with pytest.raises(ValueError, match="Expected uniforms shape"):
        tsb.sample_tokens(torch.randn(2, 10), torch.ones(2), torch.zeros(2, dtype=torch.int64),
                          torch.ones(2), torch.ones(3))


def test_sample_tokens_rejects_cpu_tensors():
    with pytest.raises(ValueError, match="CUDA tensors only"):
        tsb.sample_tokens(torch.randn(2, 10), torch.ones(2), torch.zeros(2, dtype=torch.int64),
                          torch.ones(2), torch.ones(2) * 0.5)


def test_uniforms_from_seeds_checks_lengths_and_device():
    with pytest.raises(ValueError, match="same length"):
        tsb.uniforms_from_seeds([1, 2, 3], [0, 1])
    with pytest.raises(ValueError, match="CUDA tensors only"):
        tsb.uniforms_from_seeds([1, 2], [0, 1], device="cpu")
