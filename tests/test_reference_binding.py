"""The reference-side binding, host side (no GPU): the reference's own
loader and operator names with this library installed through them.

The reference runs from its offline install (baseline/_ref, or the directory
TINYSERVER_REF names); without it these tests skip.  Only one reference
function is replaced: ``get_available_memory`` (server/model/utils.py), which
asks the GPU for free memory, returns a fixed byte count so that the
reference's ``qwen3_cache_allocator`` (server/model/patches/qwen3.py:21-64)
sizes and allocates its pool on the CPU.
"""

import pytest
import torch

from tests.common import reference_module
from tests.qwen3_tiny import tiny_model
from tinyserver_b200 import patches
from tinyserver_b200.kernels import fused, kv_cache


def test_fused_loader_runs_through_the_reference_allocator(monkeypatch):
    ref = reference_module("server.model.patches.qwen3")
    model = tiny_model(dtype=torch.float32)
    cfg = model.config
    block_bytes = 2 * cfg.num_hidden_layers * 16 * cfg.num_key_value_heads * cfg.head_dim * 4
    monkeypatch.setattr(ref, "get_available_memory", lambda utilization: 37 * block_bytes + 5)
    n = patches.fused_qwen3_model_loader(model, cfg, 0.5, 16, torch.float32, "cpu")
    assert n == 37  # the reference's own sizing rule, qwen3.py:33-42
    base = model.model
    pool = base.layers[0].self_attn.k_cache
    for i, layer in enumerate(base.layers):
        attn = layer.self_attn
        # the reference's layout: [0, i] / [1, i] views of one 6-D pool
        assert attn.k_cache.shape == (37, cfg.num_key_value_heads, 16, cfg.head_dim)
        assert attn.k_cache.untyped_storage().data_ptr() == pool.untyped_storage().data_ptr()
        assert attn.v_cache.untyped_storage().data_ptr() == pool.untyped_storage().data_ptr()
        assert "forward" in attn.__dict__, "attention forward not rebound"
        assert "forward" in layer.mlp.__dict__ and "forward" in layer.input_layernorm.__dict__
    assert "forward" in base.__dict__ and "forward" in base.embed_tokens.__dict__
    # a paged forward reads the reference's own process-global context
    ctx_mod = reference_module("server.model.inference_context")
    assert patches.qwen3._reference_context() is ctx_mod.get_inference_context


def test_fused_loader_has_the_reference_loader_signature():
    import inspect

    ref = reference_module("server.model.patches.qwen3")
    a = inspect.signature(ref.qwen3_model_loader).parameters
    b = inspect.signature(patches.fused_qwen3_model_loader).parameters
    assert list(a) == list(b)
    backend = reference_module("server.model.hf_backend")
    assert ref.qwen3_model_loader in backend.loader_by_name.values()


def test_operator_overrides_rebind_the_reference_names():
    ref = reference_module("server.model.patches.qwen3")
    originals = {n: getattr(ref, n) for n in ("apply_rotary_pos_emb", "store_kv_cache",
                                              "store_kv_cache_batched")}
    try:
        names = patches.install_operator_overrides()
        for n in originals:
            assert f"server.model.patches.qwen3.{n}" in names
        assert ref.apply_rotary_pos_emb is fused.apply_rotary_pos_emb
        assert ref.store_kv_cache is kv_cache.store_kv_cache
        assert ref.store_kv_cache_batched is kv_cache.store_kv_cache_batched
    finally:
        patches.restore_operator_overrides()
    for n, fn in originals.items():
        assert getattr(ref, n) is fn


def test_overridden_store_keeps_the_reference_validation_errors():
    """With the overrides installed, the reference module's store names raise
    the reference's ValueErrors before any device work (kv_cache.py:99-102,
    :218-234), as the reference's CPU validation tests expect."""
    ref = reference_module("server.model.patches.qwen3")
    try:
        patches.install_operator_overrides()
        k = torch.zeros(2, 4, 8)
        cache = torch.zeros(3, 2, 16, 8)
        with pytest.raises(ValueError, match="3D"):
            ref.store_kv_cache_batched(k[0], k, cache, cache, torch.zeros(4, dtype=torch.long),
                                       torch.zeros(4, dtype=torch.long))
        with pytest.raises(ValueError):
            ref.store_kv_cache(0, torch.zeros(1, dtype=torch.int32), k[0], k, cache, cache)
    finally:
        patches.restore_operator_overrides()
