"""CUDA path vs the golden vectors the reference's own code produced.

Same fixtures as tests/test_oracle_golden.py (transformers 5.5.0 Qwen3 modules
inside the reference's patched attention forward; the reference's Triton
KV-store kernels under Triton's interpreter), here run through
libqwen3fused's kernels.  Bit-exact where the contract says so (embedding,
residual add, KV placement, V rows, plain RoPE on given inputs), otherwise the
bf16/fp32 tolerance of tests/common.py.
"""

import pytest
import torch

import tinyserver_b200 as tsb
from tests.common import assert_close, expected_pool, load_golden, prefill_mapping

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(autouse=True)
def _no_device_flags():
    yield
    tsb.check_errors()


@pytest.fixture(scope="module", params=["layer_bf16.pt", "layer_f32.pt"])
def layer(request):
    return load_golden(request.param)


def _step(g, i):
    return {k: v[i] for k, v in g.items() if isinstance(v, list) and v and
            isinstance(v[0], torch.Tensor)}


def cu(t):
    return t.to(DEV)


def test_embedding(layer):
    for i in range(2):
        s = _step(layer, i)
        out = tsb.embedding(cu(s["embed.in"]), cu(layer["embed_weight"]))
        assert torch.equal(out.cpu(), s["embed.out"])


def test_input_layernorm(layer):
    for i in range(2):
        s = _step(layer, i)
        y = tsb.rms_norm(cu(s["input_layernorm.in"]), cu(layer["input_layernorm_weight"]),
                         layer["eps"])
        assert_close(y, s["input_layernorm.out"], "input_layernorm", min_exact=0.99)


def test_residual_add_post_attention_layernorm(layer):
    for i in range(2):
        s = _step(layer, i)
        y, h = tsb.fused_add_rms_norm(cu(s["o_proj.out"]), cu(s["embed.out"]),
                                      cu(layer["post_attention_layernorm_weight"]), layer["eps"])
        assert torch.equal(h.cpu(), s["post_attention_layernorm.in"])
        assert_close(y, s["post_attention_layernorm.out"], "post_attention_layernorm",
                     min_exact=0.99)


def test_residual_add_inplace(layer):
    s = _step(layer, 0)
    res = cu(s["embed.out"]).clone()
    y, h = tsb.fused_add_rms_norm(cu(s["o_proj.out"]), res,
                                  cu(layer["post_attention_layernorm_weight"]), layer["eps"],
                                  inplace=True)
    assert h.data_ptr() == res.data_ptr()
    assert torch.equal(res.cpu(), s["post_attention_layernorm.in"])


def test_q_norm_k_norm(layer):
    D = layer["head_dim"]
    for i in range(2):
        s = _step(layer, i)
        for proj, norm, w in (("q_proj", "q_norm", "q_norm_weight"),
                              ("k_proj", "k_norm", "k_norm_weight")):
            x = cu(s[proj + ".out"]).view(-1, D)
            y = tsb.rms_norm(x, cu(layer[w]), layer["eps"])
            assert_close(y, s[norm + ".out"].reshape(-1, D), norm, min_exact=0.99)


def test_rope_cos_sin(layer):
    inv = cu(layer["inv_freq"])
    for i, key in enumerate(("prefill_position_ids", "decode_position_ids")):
        s = _step(layer, i)
        cos, sin = tsb.rope_cos_sin(cu(layer[key]), inv, layer["head_dim"], s["rope.cos"].dtype)
        assert_close(cos, s["rope.cos"], "cos", min_exact=0.99)
        assert_close(sin, s["rope.sin"], "sin", min_exact=0.99)


def test_rope_cos_sin_large_positions():
    g = load_golden("rope_cos_sin.pt")
    assert torch.equal(tsb.rope_inv_freq(g["head_dim"], g["rope_theta"]), g["inv_freq"])
    for dt in (torch.float32, torch.bfloat16):
        cos, sin = tsb.rope_cos_sin(cu(g["positions"]), cu(g["inv_freq"]), g["head_dim"], dt)
        assert_close(cos[0], g[f"cos_{dt}"], f"cos {dt}", min_exact=0.99)
        assert_close(sin[0], g[f"sin_{dt}"], f"sin {dt}", min_exact=0.99)


def test_apply_rotary_pos_emb_dropin(layer):
    """Same call shape as qwen3.py:287: q/k are (1, H, T, D) transposed views."""
    for i in range(2):
        s = _step(layer, i)
        q = cu(s["q_norm.out"]).transpose(1, 2)
        k = cu(s["k_norm.out"]).transpose(1, 2)
        qo, ko = tsb.apply_rotary_pos_emb(q, k, cu(s["rope.cos"]), cu(s["rope.sin"]))
        assert qo.shape == s["rope.q_out"].shape and ko.shape == s["rope.k_out"].shape
        # the same IEEE ops on the same bf16/fp32 inputs: bit-exact
        assert torch.equal(qo.cpu(), s["rope.q_out"])
        assert torch.equal(ko.cpu(), s["rope.k_out"])


@pytest.mark.parametrize("cos_mode", ["table", "computed"])
def test_qk_norm_rope_store(layer, cos_mode):
    D, Hq, Hkv = layer["head_dim"], layer["num_q_heads"], layer["num_kv_heads"]
    B = layer["block_size"]
    pool = cu(layer["cache_before"])
    mappings = [prefill_mapping(layer["seq_lens"], layer["block_tables"], B),
                prefill_mapping([1] * len(layer["seq_lens"]), layer["block_tables"], B,
                                start_positions=layer["seq_lens"])]
    positions = [layer["prefill_position_ids"][0], layer["decode_position_ids"][0]]
    prev = layer["cache_before"]
    for i, (bm, sm) in enumerate(mappings):
        s = _step(layer, i)
        T = s["q_proj.out"].shape[1]
        q = cu(s["q_proj.out"][0]).view(T, Hq, D)
        k = cu(s["k_proj.out"][0]).view(T, Hkv, D)
        v = cu(s["v_proj.out"][0]).view(T, Hkv, D)
        kw = dict(positions=cu(positions[i]), inv_freq=cu(layer["inv_freq"])) \
            if cos_mode == "computed" else {}
        cos = cu(s["rope.cos"][0]) if cos_mode == "table" else None
        sin = cu(s["rope.sin"][0]) if cos_mode == "table" else None
        q_out, k_out = tsb.qk_norm_rope_store(
            q, k, v, cu(layer["q_norm_weight"]), cu(layer["k_norm_weight"]), layer["eps"],
            cos, sin, pool[0, 0], pool[1, 0], cu(bm), cu(sm), **kw)
        assert_close(q_out, s["rope.q_out"][0].transpose(0, 1), "q", min_exact=0.99)
        assert_close(k_out, s["rope.k_out"][0].transpose(0, 1), "k", min_exact=0.99)
        written = layer["written_prefill" if i == 0 else "written_decode"]
        rows = layer["rows_after_prefill" if i == 0 else "rows_after_decode"]
        expect = expected_pool(prev, written, rows)
        got = pool.cpu()
        assert torch.equal(got[1], expect[1]), "V pages differ"
        touched = torch.zeros(got.shape[2:5], dtype=torch.bool)
        for b, sl in written:
            touched[b, :, sl] = True
        assert torch.equal(got[0, 0][~touched], prev[0, 0][~touched]), "unwritten K slot changed"
        assert_close(got[0, 0], expect[0, 0], "k cache", min_exact=0.99)
        k_cpu = k_out.cpu()
        for t, (b, sl) in enumerate(written):
            assert torch.equal(got[0, 0, b, :, sl], k_cpu[t])
        # continue the decode step from the reference's cache state
        prev = expect
        pool.copy_(cu(expect))


def test_qk_norm_rope_without_store(layer):
    s = _step(layer, 0)
    D, Hq, Hkv = layer["head_dim"], layer["num_q_heads"], layer["num_kv_heads"]
    T = s["q_proj.out"].shape[1]
    q_out, k_out = tsb.qk_norm_rope_store(
        cu(s["q_proj.out"][0]).view(T, Hq, D), cu(s["k_proj.out"][0]).view(T, Hkv, D), None,
        cu(layer["q_norm_weight"]), cu(layer["k_norm_weight"]), layer["eps"],
        cu(s["rope.cos"][0]), cu(s["rope.sin"][0]))
    assert_close(q_out, s["rope.q_out"][0].transpose(0, 1), "q", min_exact=0.99)
    assert_close(k_out, s["rope.k_out"][0].transpose(0, 1), "k", min_exact=0.99)


def test_silu_and_mul(layer):
    for i in range(2):
        s = _step(layer, i)
        out = tsb.silu_and_mul(cu(s["gate_proj.out"]), cu(s["up_proj.out"]))
        assert_close(out, s["down_proj.in"], "silu_and_mul", min_exact=0.99)
        merged = torch.cat([cu(s["gate_proj.out"]), cu(s["up_proj.out"])], dim=-1)
        assert torch.equal(tsb.silu_and_mul(merged), out)


def test_outliers():
    g = load_golden("outliers.pt")
    y, h = tsb.fused_add_rms_norm(cu(g["x"]), cu(g["residual"]), cu(g["weight"]), g["eps"])
    assert torch.equal(h.cpu(), g["h"])
    assert_close(y, g["y"], "add_rmsnorm outliers", min_exact=0.99)
    assert_close(tsb.silu_and_mul(cu(g["gate"]), cu(g["up"])), g["act"], "silu outliers",
                 min_exact=0.99)


@pytest.mark.parametrize("entry", ["batched", "per_seq"])
def test_kv_store_reference_scenarios(entry):
    """The reference kernels' outputs on the reference tests' scenarios
    (tests/model/test_kv_cache_kernels.py:73-207 plus a bf16 permuted case)."""
    g = load_golden("kv_store.pt")
    for case in g["cases"]:
        before = torch.stack([case["cache_k_before"], case["cache_v_before"]])[:, None]
        written = list(zip(case["block_mapping"].tolist(), case["slot_mapping"].tolist()))
        expect = expected_pool(before, written, case["written_rows"])
        kc, vc = cu(case["cache_k_before"]), cu(case["cache_v_before"])
        if entry == "batched":
            tsb.store_kv_cache_batched(cu(torch.cat(case["k_srcs"], 1)),
                                       cu(torch.cat(case["v_srcs"], 1)), kc, vc,
                                       cu(case["block_mapping"]), cu(case["slot_mapping"]))
        else:
            for sq, ks, vs in zip(case["seqs"], case["k_srcs"], case["v_srcs"]):
                tsb.store_kv_cache(sq["start_pos"], cu(torch.tensor(sq["block_table"],
                                                                    dtype=torch.int32)),
                                   cu(ks), cu(vs), kc, vc)
        assert torch.equal(kc.cpu(), expect[0, 0]), case["name"]
        assert torch.equal(vc.cpu(), expect[1, 0]), case["name"]
