"""Drop-in installation, host side (no GPU): which forwards are rebound, the
operator-name overrides, and that the installed model fails loudly on CPU
tensors instead of falling back to torch."""

import pytest
import torch

from tests.qwen3_tiny import tiny_model
from tinyserver_b200 import patches


def test_install_rebinds_every_module_forward():
    from transformers.models.qwen3.modeling_qwen3 import (Qwen3DecoderLayer, Qwen3MLP,
                                                          Qwen3RMSNorm)

    model = tiny_model(dtype=torch.float32)
    patches.install_fused(model, paged=False)
    base = model.model
    kinds = {Qwen3RMSNorm: 0, Qwen3MLP: 0, Qwen3DecoderLayer: 0}
    for mod in base.modules():
        for cls in kinds:
            if isinstance(mod, cls):
                assert "forward" in mod.__dict__, f"{cls.__name__} not rebound"
                kinds[cls] += 1
    L = model.config.num_hidden_layers
    # input/post norms per layer, q_norm/k_norm per layer, the final norm
    assert kinds[Qwen3RMSNorm] == 4 * L + 1
    assert kinds[Qwen3MLP] == L and kinds[Qwen3DecoderLayer] == L
    assert "forward" in base.embed_tokens.__dict__
    # attention stays the model's own when not paged
    assert all("forward" not in layer.self_attn.__dict__ for layer in base.layers)


def test_paged_install_needs_a_cache():
    model = tiny_model(dtype=torch.float32)
    with pytest.raises(ValueError, match="k_cache"):
        patches.install_fused(model, paged=True, context=lambda: None, attention=object())


def test_paged_install_rebinds_attention():
    model = tiny_model(dtype=torch.float32)
    patches.allocate_kv_cache(model, num_blocks=8, block_size=16, dtype=torch.float32,
                              device="cpu")
    patches.install_fused(model, context=lambda: None, attention=object())
    assert all("forward" in layer.self_attn.__dict__ for layer in model.model.layers)
    assert "forward" in model.model.__dict__  # the fused layer loop
    with pytest.raises(ValueError, match="use_cache=False"):
        model.model(input_ids=torch.zeros(1, 4, dtype=torch.long), use_cache=True)
    k0 = model.model.layers[0].self_attn.k_cache
    assert k0.shape == (8, model.config.num_key_value_heads, 16, model.config.head_dim)


def test_installed_model_refuses_cpu_tensors():
    model = tiny_model(dtype=torch.float32)
    patches.install_fused(model, paged=False)
    ids = torch.randint(0, 512, (1, 8))
    with pytest.raises(ValueError, match="CUDA tensors only"):
        model(input_ids=ids, position_ids=torch.arange(8)[None], use_cache=False)


def test_operator_overrides_rebind_and_restore():
    import transformers.models.qwen3.modeling_qwen3 as hf

    from tinyserver_b200.kernels import fused

    original = hf.apply_rotary_pos_emb
    try:
        names = patches.install_operator_overrides()
        assert "transformers.models.qwen3.modeling_qwen3.apply_rotary_pos_emb" in names
        assert hf.apply_rotary_pos_emb is fused.apply_rotary_pos_emb
    finally:
        patches.restore_operator_overrides()
    assert hf.apply_rotary_pos_emb is original


def test_fused_forward_drops_the_cached_mapping_of_a_reused_context():
    """A context object reused across forwards: the fused model forward drops
    the batch mapping cached on it before its layers run, so a stale mapping
    (same position_ids address, different sequences) is never served."""
    from tests.qwen3_tiny import Context

    model = tiny_model(dtype=torch.float32)
    patches.allocate_kv_cache(model, num_blocks=8, block_size=16, dtype=torch.float32,
                              device="cpu")
    ctx = Context(mode="prefill", sequences=[{"num_tokens": 4, "block_table": [0]}])
    ctx._tinyserver_b200_mapping = "stale"
    patches.install_fused(model, context=lambda: ctx, attention=object())
    with pytest.raises(ValueError, match="CUDA tensors only"):  # the first op needs a GPU
        model.model(input_ids=torch.zeros(1, 4, dtype=torch.long), use_cache=False)
    assert ctx._tinyserver_b200_mapping is None
