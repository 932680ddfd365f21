"""torch.ops.qwen3fused on the GPU: every op through torch.library.opcheck
(the schema's declared writes against what the launch really mutates, and
the fake implementation's shapes, dtypes and strides against the real
outputs), equal to the direct function, and a decoder-layer slice under
torch.compile(fullgraph=True) equal to the same ops run eagerly."""

import pytest
import torch

import tinyserver_b200 as tsb

pytestmark = pytest.mark.gpu
Q = torch.ops.qwen3fused
DEV = "cuda"
BF = torch.bfloat16
CHECKS = ("test_schema", "test_faketensor")


def _g(seed):
    return torch.Generator(device=DEV).manual_seed(seed)


def _rand(*shape, seed, dtype=BF):
    return torch.randn(*shape, generator=_g(seed), device=DEV).to(dtype)


def _layer_inputs(T=40, H=256, Hq=4, Hkv=2, D=128, I=512, N=16, B=16, seed=0):
    g = _g(seed)
    pos = torch.randint(0, N * B // 2, (T,), generator=g, device=DEV)
    perm = torch.randperm(N * B, generator=g, device=DEV)[:T]
    return dict(
        ids=torch.randint(0, 1000, (T,), generator=g, device=DEV),
        table=_rand(1000, H, seed=seed + 1), x_attn=_rand(T, H, seed=seed + 2),
        w_in=1 + 0.02 * _rand(H, seed=seed + 3), qkv=_rand(T, (Hq + 2 * Hkv) * D, seed=seed + 4),
        qw=1 + 0.02 * _rand(D, seed=seed + 5), kw=1 + 0.02 * _rand(D, seed=seed + 6),
        pos=pos, inv=tsb.rope_inv_freq(D, 1e6, DEV),
        kc=_rand(N, Hkv, B, D, seed=seed + 7), vc=_rand(N, Hkv, B, D, seed=seed + 8),
        bm=perm // B, sm=perm % B, w_post=1 + 0.02 * _rand(H, seed=seed + 9),
        x_mlp=_rand(T, H, seed=seed + 10), gate_up=_rand(T, 2 * I, seed=seed + 11),
        dims=(T, H, Hq, Hkv, D, I))


def _qkv_views(qkv, T, Hq, Hkv, D):
    return (qkv[:, :Hq * D].view(T, Hq, D), qkv[:, Hq * D:(Hq + Hkv) * D].view(T, Hkv, D),
            qkv[:, (Hq + Hkv) * D:].view(T, Hkv, D))


def test_fused_ops_pass_opcheck_and_equal_the_direct_functions():
    a = _layer_inputs()
    T, H, Hq, Hkv, D, I = a["dims"]
    torch.library.opcheck(Q.embedding.default, (a["ids"], a["table"]), test_utils=CHECKS)
    assert torch.equal(Q.embedding(a["ids"], a["table"]), tsb.embedding(a["ids"], a["table"]))
    torch.library.opcheck(Q.rms_norm.default, (a["x_attn"], a["w_in"], 1e-6), test_utils=CHECKS)
    assert torch.equal(Q.rms_norm(a["x_attn"], a["w_in"], 1e-6),
                       tsb.rms_norm(a["x_attn"], a["w_in"], 1e-6))
    args = (a["x_attn"], a["x_mlp"], a["w_in"], 1e-6)
    torch.library.opcheck(Q.fused_add_rms_norm.default, args, test_utils=CHECKS)
    for got, want in zip(Q.fused_add_rms_norm(*args), tsb.fused_add_rms_norm(*args)):
        assert torch.equal(got, want)
    torch.library.opcheck(Q.silu_and_mul.default, (a["gate_up"],), test_utils=CHECKS)
    assert torch.equal(Q.silu_and_mul(a["gate_up"]), tsb.silu_and_mul(a["gate_up"]))
    cargs = (a["pos"], a["inv"], D, BF)
    torch.library.opcheck(Q.rope_cos_sin.default, cargs, test_utils=CHECKS)
    cos, sin = Q.rope_cos_sin(*cargs)
    rc, rs = tsb.rope_cos_sin(*cargs)
    assert torch.equal(cos, rc) and torch.equal(sin, rs)
    tsb.check_errors()


def test_store_ops_declare_their_cache_writes_and_equal_the_direct_functions():
    a = _layer_inputs(seed=20)
    T, H, Hq, Hkv, D, I = a["dims"]
    cos, sin = tsb.rope_cos_sin(a["pos"], a["inv"], D, BF)
    q, k, v = _qkv_views(a["qkv"], T, Hq, Hkv, D)
    # opcheck's schema test sees the caches change: the writes are declared
    torch.library.opcheck(Q.qk_norm_rope_store.default,
                          (q, k, v, a["qw"], a["kw"], 1e-6, cos, sin, a["kc"].clone(),
                           a["vc"].clone(), a["bm"], a["sm"]), test_utils=CHECKS)
    kc1, vc1, kc2, vc2 = a["kc"].clone(), a["vc"].clone(), a["kc"].clone(), a["vc"].clone()
    got = Q.qk_norm_rope_store(q, k, v, a["qw"], a["kw"], 1e-6, cos, sin, kc1, vc1, a["bm"],
                               a["sm"])
    want = tsb.qk_norm_rope_store(q, k, v, a["qw"], a["kw"], 1e-6, cos, sin, kc2, vc2, a["bm"],
                                  a["sm"])
    assert torch.equal(got[0], want[0]) and torch.equal(got[1], want[1])
    assert torch.equal(kc1, kc2) and torch.equal(vc1, vc2)
    ks, vs = k.transpose(0, 1).contiguous(), v.transpose(0, 1).contiguous()
    torch.library.opcheck(Q.store_kv_cache_batched.default,
                          (ks, vs, a["kc"].clone(), a["vc"].clone(), a["bm"], a["sm"]),
                          test_utils=CHECKS)
    kc1, vc1, kc2, vc2 = a["kc"].clone(), a["vc"].clone(), a["kc"].clone(), a["vc"].clone()
    Q.store_kv_cache_batched(ks, vs, kc1, vc1, a["bm"], a["sm"])
    tsb.store_kv_cache_batched(ks, vs, kc2, vc2, a["bm"], a["sm"])
    assert torch.equal(kc1, kc2) and torch.equal(vc1, vc2)
    bt = torch.tensor([3, 7, 1], dtype=torch.int32, device=DEV)
    ks5, vs5 = ks[:, :5].contiguous(), vs[:, :5].contiguous()
    torch.library.opcheck(Q.store_kv_cache.default,
                          (13, bt, ks5, vs5, a["kc"].clone(), a["vc"].clone()), test_utils=CHECKS)
    kc1, vc1, kc2, vc2 = a["kc"].clone(), a["vc"].clone(), a["kc"].clone(), a["vc"].clone()
    Q.store_kv_cache(13, bt, ks5, vs5, kc1, vc1)
    tsb.store_kv_cache(13, bt, ks5, vs5, kc2, vc2)
    assert torch.equal(kc1, kc2) and torch.equal(vc1, vc2)
    tsb.check_errors()


@pytest.mark.parametrize("unsqueeze_dim", [1, 2])
@pytest.mark.parametrize("batch", [1, 2])
def test_rotary_op_passes_opcheck(unsqueeze_dim, batch):
    T, Hq, Hkv, D = 24, 4, 2, 128
    shape_q = (batch, Hq, T, D) if unsqueeze_dim == 1 else (batch, T, Hq, D)
    shape_k = (batch, Hkv, T, D) if unsqueeze_dim == 1 else (batch, T, Hkv, D)
    q, k = _rand(*shape_q, seed=31), _rand(*shape_k, seed=32)
    pos = torch.arange(T, device=DEV).expand(batch, T)
    cos, sin = tsb.rope_cos_sin(pos, tsb.rope_inv_freq(D, 1e6, DEV), D, BF)
    args = (q, k, cos, sin, unsqueeze_dim)
    torch.library.opcheck(Q.apply_rotary_pos_emb.default, args, test_utils=CHECKS)
    for got, want in zip(Q.apply_rotary_pos_emb(*args), tsb.apply_rotary_pos_emb(*args)):
        assert torch.equal(got, want) and got.stride() == want.stride()


def test_mapping_attention_and_sampling_ops_pass_opcheck():
    cu = torch.tensor([0, 5, 12], dtype=torch.int32, device=DEV)
    pos = torch.cat([torch.arange(3, 8), torch.arange(20, 27)]).to(DEV)
    bt = torch.tensor([[4, 9, 0, 0], [1, 2, 3, 5]], dtype=torch.int32, device=DEV)
    torch.library.opcheck(Q.build_slot_mapping.default, (cu, pos, bt, 16), test_utils=CHECKS)
    got, want = Q.build_slot_mapping(cu, pos, bt, 16), tsb.build_slot_mapping(cu, pos, bt, 16)
    assert all(torch.equal(x, y) for x, y in zip(got, want))

    S, Hq, Hkv, D, B = 3, 8, 2, 128, 16
    query, kc, vc = _rand(S, Hq, D, seed=41), _rand(12, Hkv, B, D, seed=42), \
        _rand(12, Hkv, B, D, seed=43)
    btab = torch.arange(12, dtype=torch.int32, device=DEV).view(S, 4)
    lens = torch.tensor([5, 40, 64], dtype=torch.int32, device=DEV)
    args = (query, kc, vc, btab, B, lens)
    torch.library.opcheck(Q.paged_attention_forward.default, args, test_utils=CHECKS)
    assert torch.equal(Q.paged_attention_forward(*args), tsb.paged_attention_forward(*args))

    q, k, v = _rand(150, 8, 128, seed=44), _rand(150, 2, 128, seed=45), _rand(150, 2, 128, seed=46)
    cuq = torch.tensor([0, 60, 150], dtype=torch.int32, device=DEV)
    args = (q, k, v, cuq, cuq, 90, 90, True, None)
    torch.library.opcheck(Q.flash_attn_varlen_func.default, args, test_utils=CHECKS)
    assert torch.equal(Q.flash_attn_varlen_func(*args), tsb.flash_attn_varlen_func(*args))

    logits = _rand(4, 5000, seed=47)
    t = torch.tensor([0.0, 0.7, 1.0, 1.3], device=DEV)
    topk = torch.tensor([0, 20, 0, 100], device=DEV)
    topp = torch.tensor([1.0, 0.9, 0.95, 1.0], device=DEV)
    u = torch.tensor([0.1, 0.5, 0.9, 0.3], device=DEV)
    args = (logits, t, topk, topp, u)
    torch.library.opcheck(Q.sample_tokens.default, args, test_utils=CHECKS)
    assert torch.equal(Q.sample_tokens(*args), tsb.sample_tokens(*args))
    seeds = torch.tensor([1, 2, 3, 4], device=DEV)
    steps = torch.tensor([0, 5, 9, 2], device=DEV)
    args = (logits, t, topk, topp, seeds, steps)
    torch.library.opcheck(Q.sample_tokens_seeded.default, args, test_utils=CHECKS)
    assert torch.equal(Q.sample_tokens_seeded(*args), tsb.sample_tokens_seeded(*args))
    torch.library.opcheck(Q.uniforms_from_seeds.default, (seeds, steps), test_utils=CHECKS)
    assert torch.equal(Q.uniforms_from_seeds(seeds, steps), tsb.uniforms_from_seeds(seeds, steps))
    tsb.check_errors()


def test_compiled_layer_slice_equals_eager():
    """embedding -> add + RMSNorm -> q/k norm + RoPE + store -> add + RMSNorm ->
    SiLU-and-mul under torch.compile(fullgraph=True): the same outputs and the
    same cache contents as the ops run eagerly."""
    a = _layer_inputs(seed=60)
    T, H, Hq, Hkv, D, I = a["dims"]

    def layer(ids, table, x_attn, w_in, qkv, qw, kw, pos, inv, kc, vc, bm, sm, w_post, x_mlp,
              gate_up):
        x0 = Q.embedding(ids, table)
        y, h = Q.fused_add_rms_norm(x_attn, x0, w_in, 1e-6)
        cos, sin = Q.rope_cos_sin(pos, inv, D, BF)
        q, k, v = _qkv_views(qkv, T, Hq, Hkv, D)
        qo, ko = Q.qk_norm_rope_store(q, k, v, qw, kw, 1e-6, cos, sin, kc, vc, bm, sm)
        y2, h2 = Q.fused_add_rms_norm(x_mlp, h, w_post, 1e-6)
        return y, qo, ko, y2, h2, Q.silu_and_mul(gate_up)

    def run(fn):
        kc, vc = a["kc"].clone(), a["vc"].clone()
        outs = fn(a["ids"], a["table"], a["x_attn"], a["w_in"], a["qkv"], a["qw"], a["kw"],
                  a["pos"], a["inv"], kc, vc, a["bm"], a["sm"], a["w_post"], a["x_mlp"],
                  a["gate_up"])
        torch.cuda.synchronize()
        return outs, kc, vc

    torch._dynamo.reset()
    eager, kce, vce = run(layer)
    compiled, kcc, vcc = run(torch.compile(layer, fullgraph=True))
    for i, (x, y) in enumerate(zip(eager, compiled)):
        assert torch.equal(x, y), f"output {i}"
    assert torch.equal(kce, kcc) and torch.equal(vce, vcc), "cache contents"
    tsb.check_errors()
