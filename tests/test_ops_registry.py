"""The torch.library registration of the path's operators (torch.ops.qwen3fused),
checked without a GPU: every op's schema (the stores declare their cache
writes), and every fake implementation under FakeTensorMode on fake CUDA
tensors, shape, dtype and stride, including graphs traced through several ops.
The real launches are checked against the fakes in test_gpu_ops_registry.py."""

import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode
from torch.fx.experimental.proxy_tensor import make_fx

import tinyserver_b200  # noqa: F401  (registers torch.ops.qwen3fused)
from tinyserver_b200 import ops

Q = torch.ops.qwen3fused
BF = torch.bfloat16


def _schema(name):
    return getattr(Q, name).default._schema


def test_every_op_is_registered_under_the_namespace():
    for name in ops.OPS:
        assert hasattr(Q, name), name
        assert str(_schema(name)).startswith(f"qwen3fused::{name}(")


@pytest.mark.parametrize("name,mutated", [
    ("store_kv_cache_batched", {"k_cache", "v_cache"}),
    ("store_kv_cache", {"k_cache", "v_cache"}),
    ("qk_norm_rope_store", {"k_cache", "v_cache"}),
    ("rms_norm", set()), ("fused_add_rms_norm", set()), ("embedding", set()),
    ("silu_and_mul", set()), ("paged_attention_forward", set()),
    ("flash_attn_varlen_func", set()), ("sample_tokens", set()),
])
def test_schemas_declare_exactly_the_in_place_cache_writes(name, mutated):
    s = _schema(name)
    written = {a.name for a in s.arguments if a.alias_info is not None and a.alias_info.is_write}
    assert written == mutated
    assert all(r.alias_info is None for r in s.returns), "outputs never alias inputs"


def test_reference_signatures_are_kept():
    # store_kv_cache(start_position, block_table, k_src, v_src, k_cache, v_cache)
    assert [a.name for a in _schema("store_kv_cache").arguments] == [
        "start_position", "block_table", "k_src", "v_src", "k_cache", "v_cache"]
    assert [a.name for a in _schema("store_kv_cache_batched").arguments] == [
        "k_src", "v_src", "k_cache", "v_cache", "block_mapping", "slot_mapping"]
    assert [a.name for a in _schema("apply_rotary_pos_emb").arguments] == [
        "q", "k", "cos", "sin", "unsqueeze_dim"]


def _fake(*shape, dtype=BF):
    return torch.empty(*shape, dtype=dtype, device="cuda")


def test_fake_outputs_of_the_fused_ops():
    T, H, Hq, Hkv, D, I = 48, 256, 4, 2, 128, 512
    with FakeTensorMode():
        ids = _fake(2, 24, dtype=torch.int64)
        table = _fake(1000, H)
        assert Q.embedding(ids, table).shape == (2, 24, H)
        x, w = _fake(T, H), _fake(H)
        y = Q.rms_norm(x, w, 1e-6)
        assert y.shape == x.shape and y.dtype == BF and y.is_contiguous()
        y, h = Q.fused_add_rms_norm(x, _fake(T, H), w, 1e-6)
        assert y.shape == h.shape == (T, H)
        assert Q.silu_and_mul(_fake(T, 2 * I)).shape == (T, I)
        assert Q.silu_and_mul(_fake(T, I), _fake(T, I)).shape == (T, I)
        pos = _fake(T, dtype=torch.int64)
        cos, sin = Q.rope_cos_sin(pos, _fake(D // 2, dtype=torch.float32), D, BF)
        assert cos.shape == sin.shape == (T, D) and cos.dtype == BF
        qkv = _fake(T, (Hq + 2 * Hkv) * D)
        q = qkv[:, :Hq * D].view(T, Hq, D)
        k = qkv[:, Hq * D:(Hq + Hkv) * D].view(T, Hkv, D)
        v = qkv[:, (Hq + Hkv) * D:].view(T, Hkv, D)
        kc, vc = _fake(8, Hkv, 16, D), _fake(8, Hkv, 16, D)
        bm = sm = _fake(T, dtype=torch.int64)
        qo, ko = Q.qk_norm_rope_store(q, k, v, _fake(D), _fake(D), 1e-6, cos, sin, kc, vc, bm,
                                      sm)
        assert qo.shape == (T, Hq, D) and ko.shape == (T, Hkv, D)
        assert Q.store_kv_cache_batched(k.transpose(0, 1), v.transpose(0, 1), kc, vc, bm,
                                        sm) is None
        bt = _fake(4, dtype=torch.int32)
        assert Q.store_kv_cache(5, bt, _fake(Hkv, 3, D), _fake(Hkv, 3, D), kc, vc) is None
        bmo, smo = Q.build_slot_mapping(_fake(3, dtype=torch.int32), pos,
                                        _fake(2, 4, dtype=torch.int32), 16)
        assert bmo.shape == smo.shape == (T,) and bmo.dtype == torch.int64


@pytest.mark.parametrize("unsqueeze_dim", [1, 2])
@pytest.mark.parametrize("batch", [1, 3])
def test_fake_rotary_matches_the_real_ops_layout(unsqueeze_dim, batch):
    """The real op returns token-major memory: for (B, H, T, D) inputs a
    transposed view when B = 1.  The fake gives the same strides."""
    T, Hq, Hkv, D = 10, 4, 2, 64
    with FakeTensorMode():
        if unsqueeze_dim == 1:
            q, k = _fake(batch, Hq, T, D), _fake(batch, Hkv, T, D)
        else:
            q, k = _fake(batch, T, Hq, D), _fake(batch, T, Hkv, D)
        qo, ko = Q.apply_rotary_pos_emb(q, k, _fake(batch, T, D), _fake(batch, T, D),
                                        unsqueeze_dim)
        assert qo.shape == q.shape and ko.shape == k.shape
        if unsqueeze_dim == 1 and batch == 1:
            assert qo.stride()[1:] == (D, Hq * D, 1)  # (H, T, D) over token-major rows
        else:
            assert qo.is_contiguous()


def test_fake_outputs_of_attention_and_sampling():
    with FakeTensorMode():
        qd = _fake(6, 8, 128)
        kc = _fake(20, 2, 16, 128)
        out = Q.paged_attention_forward(qd, kc, kc, _fake(6, 4, dtype=torch.int32), 16,
                                        _fake(6, dtype=torch.int32))
        assert out.shape == qd.shape and out.dtype == BF
        q, k = _fake(100, 8, 128), _fake(100, 2, 128)
        cu = _fake(3, dtype=torch.int32)
        o = Q.flash_attn_varlen_func(q, k, k, cu, cu, 64, 64, True, None)
        assert o.shape == q.shape
        logits = _fake(5, 1000)
        f32, i64 = torch.float32, torch.int64
        tok = Q.sample_tokens(logits, _fake(5, dtype=f32), _fake(5, dtype=i64),
                              _fake(5, dtype=f32), _fake(5, dtype=f32))
        assert tok.shape == (5,) and tok.dtype == i64
        tok = Q.sample_tokens_seeded(logits, _fake(5, dtype=f32), _fake(5, dtype=i64),
                                     _fake(5, dtype=f32), _fake(5, dtype=i64), _fake(5, dtype=i64))
        assert tok.shape == (5,) and tok.dtype == i64
        u = Q.uniforms_from_seeds(_fake(5, dtype=i64), _fake(5, dtype=i64))
        assert u.shape == (5,) and u.dtype == f32


def test_a_layer_slice_traces_to_single_op_nodes():
    """A graph traced through the ops on fake CUDA tensors holds each as one
    node, the cache store included, in program order."""
    T, H, Hq, Hkv, D, I = 32, 256, 4, 2, 128, 512

    def layer(ids, table, x_attn, w_in, qkv, qw, kw, cos, sin, kc, vc, bm, sm, w_post, x_mlp,
              gate_up):
        x0 = Q.embedding(ids, table)
        y, h = Q.fused_add_rms_norm(x_attn, x0, w_in, 1e-6)
        q = qkv[:, :Hq * D].view(T, Hq, D)
        k = qkv[:, Hq * D:(Hq + Hkv) * D].view(T, Hkv, D)
        v = qkv[:, (Hq + Hkv) * D:].view(T, Hkv, D)
        qo, ko = Q.qk_norm_rope_store(q, k, v, qw, kw, 1e-6, cos, sin, kc, vc, bm, sm)
        y2, h2 = Q.fused_add_rms_norm(x_mlp, h, w_post, 1e-6)
        return y, qo, y2, h2, Q.silu_and_mul(gate_up)

    with FakeTensorMode():
        args = (_fake(T, dtype=torch.int64), _fake(1000, H), _fake(T, H), _fake(H),
                _fake(T, (Hq + 2 * Hkv) * D), _fake(D), _fake(D), _fake(T, D), _fake(T, D),
                _fake(8, Hkv, 16, D), _fake(8, Hkv, 16, D), _fake(T, dtype=torch.int64),
                _fake(T, dtype=torch.int64), _fake(H), _fake(T, H), _fake(T, 2 * I))
        gm = make_fx(layer, tracing_mode="fake")(*args)
    calls = [str(n.target) for n in gm.graph.nodes
             if n.op == "call_function" and str(n.target).startswith("qwen3fused.")]
    assert calls == ["qwen3fused.embedding.default", "qwen3fused.fused_add_rms_norm.default",
                     "qwen3fused.qk_norm_rope_store.default",
                     "qwen3fused.fused_add_rms_norm.default", "qwen3fused.silu_and_mul.default"]


def test_real_ops_keep_the_no_cpu_fallback_rule():
    """Through the dispatcher too, a CPU tensor is refused, not computed."""
    x, w = torch.randn(4, 64, dtype=BF), torch.ones(64, dtype=BF)
    with pytest.raises((RuntimeError, ValueError)):
        Q.rms_norm(x, w, 1e-6)
