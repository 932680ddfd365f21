"""Pin the CPU oracle against the golden vectors the reference's own code wrote.

The fixtures come from tests/golden/make_golden.py: transformers 5.5.0's Qwen3
modules inside the reference's patched attention forward, and the reference's
Triton KV-store kernels run by Triton's CPU interpreter.  Passing here is what
lets the GPU tests use the oracle as the reference at sizes no fixture holds.
"""

import pytest
import torch

from oracle import oracle
from tests.common import assert_close, expected_pool, load_golden, prefill_mapping


@pytest.fixture(scope="module", params=["layer_bf16.pt", "layer_f32.pt"])
def layer(request):
    return load_golden(request.param)


def _step(g, i):
    """Per-step view of the captures: i = 0 prefill, 1 decode."""
    return {k: v[i] for k, v in g.items() if isinstance(v, list) and v and
            isinstance(v[0], torch.Tensor)}


def test_embedding_bit_exact(layer):
    for i in range(2):
        s = _step(layer, i)
        out = oracle.embedding(s["embed.in"], layer["embed_weight"])
        assert torch.equal(out, s["embed.out"][0])


def test_oracle_rejects_out_of_range_token(layer):
    ids = torch.tensor([0, layer["embed_weight"].shape[0]])
    with pytest.raises(IndexError):
        oracle.embedding(ids, layer["embed_weight"])


def test_input_layernorm(layer):
    for i in range(2):
        s = _step(layer, i)
        y = oracle.rmsnorm(s["input_layernorm.in"][0], layer["input_layernorm_weight"],
                           layer["eps"])
        assert_close(y, s["input_layernorm.out"][0], "input_layernorm", min_exact=0.99)


def test_residual_add_and_post_attention_layernorm(layer):
    for i in range(2):
        s = _step(layer, i)
        # layer 0: residual = embedding output (HF:315), x = o_proj output (HF:327)
        y, h = oracle.add_rmsnorm(s["o_proj.out"][0], s["embed.out"][0],
                                  layer["post_attention_layernorm_weight"], layer["eps"])
        assert torch.equal(h, s["post_attention_layernorm.in"][0])
        assert_close(y, s["post_attention_layernorm.out"][0], "post_attention_layernorm",
                     min_exact=0.99)


def test_q_norm_k_norm(layer):
    D = layer["head_dim"]
    for i in range(2):
        s = _step(layer, i)
        for proj, norm, w in (("q_proj", "q_norm", "q_norm_weight"),
                              ("k_proj", "k_norm", "k_norm_weight")):
            x = s[proj + ".out"][0].reshape(-1, D)
            y = oracle.rmsnorm(x, layer[w], layer["eps"])
            assert_close(y, s[norm + ".out"][0].reshape(-1, D), norm, min_exact=0.99)


def test_rotary_cos_sin(layer):
    for i, pos_key in enumerate(("prefill_position_ids", "decode_position_ids")):
        s = _step(layer, i)
        dt = s["rope.cos"].dtype
        cos, sin = oracle.rope_cos_sin(layer[pos_key], layer["inv_freq"], layer["head_dim"], dt)
        assert_close(cos, s["rope.cos"][0], "cos", min_exact=0.99)
        assert_close(sin, s["rope.sin"][0], "sin", min_exact=0.99)


def test_rope_cos_sin_large_positions():
    g = load_golden("rope_cos_sin.pt")
    ref_inv = oracle.rope_inv_freq(g["head_dim"], g["rope_theta"])
    assert torch.equal(ref_inv, g["inv_freq"])
    for dt in (torch.float32, torch.bfloat16):
        cos, sin = oracle.rope_cos_sin(g["positions"], g["inv_freq"], g["head_dim"], dt)
        assert_close(cos, g[f"cos_{dt}"], f"cos {dt}", min_exact=0.99)
        assert_close(sin, g[f"sin_{dt}"], f"sin {dt}", min_exact=0.99)


def _qk_inputs(layer, s):
    T = s["q_proj.out"].shape[1]
    D, Hq, Hkv = layer["head_dim"], layer["num_q_heads"], layer["num_kv_heads"]
    q = s["q_proj.out"][0].view(T, Hq, D)
    k = s["k_proj.out"][0].view(T, Hkv, D)
    v = s["v_proj.out"][0].view(T, Hkv, D)
    return q, k, v


def test_qk_norm_rope_store_prefill_and_decode(layer):
    pool = layer["cache_before"].clone()
    B = layer["block_size"]
    bts = layer["block_tables"]
    lens = layer["seq_lens"]
    mappings = [prefill_mapping(lens, bts, B),
                prefill_mapping([1] * len(lens), bts, B, start_positions=lens)]
    for i, (bm, sm) in enumerate(mappings):
        s = _step(layer, i)
        q, k, v = _qk_inputs(layer, s)
        q_out, k_out = oracle.qk_norm_rope_store(
            q, k, v, layer["q_norm_weight"], layer["k_norm_weight"], layer["eps"],
            s["rope.cos"][0], s["rope.sin"][0], pool[0, 0], pool[1, 0], bm, sm)
        assert_close(q_out, s["rope.q_out"][0].transpose(0, 1), "rope q", min_exact=0.99)
        assert_close(k_out, s["rope.k_out"][0].transpose(0, 1), "rope k", min_exact=0.99)
        written = layer["written_prefill" if i == 0 else "written_decode"]
        rows = layer["rows_after_prefill" if i == 0 else "rows_after_decode"]
        prev = layer["cache_before"] if i == 0 else expected_pool(
            layer["cache_before"], layer["written_prefill"], layer["rows_after_prefill"])
        expect = expected_pool(prev, written, rows)
        # V rows are copies and every unwritten row is untouched: bit-exact.
        assert torch.equal(pool[1], expect[1])
        touched = torch.zeros(pool.shape[2:5], dtype=torch.bool)
        for b, sl in written:
            touched[b, :, sl] = True
        assert torch.equal(pool[0, 0][~touched], prev[0, 0][~touched])
        # K rows hold the rotated K: the oracle's own k_out, bit for bit, and
        # the reference's within tolerance.
        assert_close(pool[0, 0], expect[0, 0], "k cache", min_exact=0.99)
        for t, (b, sl) in enumerate(written):
            assert torch.equal(pool[0, 0, b, :, sl], k_out[t])
        # carry the reference's state forward so the decode step starts from it
        pool = expect.clone()


def test_plain_rope_without_norm(layer):
    s = _step(layer, 0)
    T = s["q_norm.out"].shape[1]
    q_out, k_out = oracle.qk_norm_rope_store(
        s["q_norm.out"][0], s["k_norm.out"][0], None, None, None, layer["eps"],
        s["rope.cos"][0], s["rope.sin"][0])
    assert torch.equal(q_out, s["rope.q_out"][0].transpose(0, 1))
    assert torch.equal(k_out, s["rope.k_out"][0].transpose(0, 1))
    assert q_out.shape[0] == T


def test_silu_and_mul(layer):
    for i in range(2):
        s = _step(layer, i)
        out = oracle.silu_and_mul(s["gate_proj.out"][0], s["up_proj.out"][0])
        assert_close(out, s["down_proj.in"][0], "silu_and_mul", min_exact=0.99)


def test_silu_and_mul_merged_layout(layer):
    s = _step(layer, 0)
    g, u = s["gate_proj.out"][0], s["up_proj.out"][0]
    merged = torch.cat([g, u], dim=-1)
    I = g.shape[-1]
    out = oracle.silu_and_mul(merged[:, :I], merged[:, I:])
    assert torch.equal(out, oracle.silu_and_mul(g, u))


def test_outliers():
    g = load_golden("outliers.pt")
    y, h = oracle.add_rmsnorm(g["x"], g["residual"], g["weight"], g["eps"])
    assert torch.equal(h, g["h"])
    assert_close(y, g["y"], "add_rmsnorm outliers", min_exact=0.99)
    act = oracle.silu_and_mul(g["gate"], g["up"])
    assert_close(act, g["act"], "silu outliers", min_exact=0.99)


def test_kv_store_reference_kernels():
    g = load_golden("kv_store.pt")
    for case in g["cases"]:
        before = torch.stack([case["cache_k_before"], case["cache_v_before"]])[:, None]
        written = list(zip(case["block_mapping"].tolist(), case["slot_mapping"].tolist()))
        expect = expected_pool(before, written, case["written_rows"])
        # batched store
        kc, vc = case["cache_k_before"].clone(), case["cache_v_before"].clone()
        oracle.kv_store_batched(torch.cat(case["k_srcs"], 1), torch.cat(case["v_srcs"], 1),
                                kc, vc, case["block_mapping"], case["slot_mapping"])
        assert torch.equal(kc, expect[0, 0]), case["name"]
        assert torch.equal(vc, expect[1, 0]), case["name"]
        # per-sequence store
        kc, vc = case["cache_k_before"].clone(), case["cache_v_before"].clone()
        for sq, ks, vs in zip(case["seqs"], case["k_srcs"], case["v_srcs"]):
            oracle.kv_store_seq(sq["start_pos"], torch.tensor(sq["block_table"], dtype=torch.int32),
                                ks, vs, kc, vc)
        assert torch.equal(kc, expect[0, 0]), case["name"]
        assert torch.equal(vc, expect[1, 0]), case["name"]


def test_kv_store_rejects_out_of_range_slot():
    k = torch.randn(2, 3, 8)
    kc = torch.zeros(2, 2, 4, 8)
    vc = torch.zeros_like(kc)
    with pytest.raises(IndexError):
        oracle.kv_store_batched(k, k, kc, vc, torch.tensor([0, 1, 2]), torch.tensor([0, 1, 2]))
    with pytest.raises(IndexError):
        oracle.kv_store_batched(k, k, kc, vc, torch.tensor([0, 1, 1]), torch.tensor([0, 1, 4]))
    assert not kc.any() and not vc.any()


def test_paged_attention_decode_matches_reference_kernel():
    """The oracle against the reference's own Triton decode attention (run
    under Triton's interpreter when the fixture was made)."""
    g = load_golden("paged_attention.pt")
    for c in g["cases"]:
        out = oracle.paged_attention_decode(c["query"], c["k_cache"], c["v_cache"],
                                            c["block_tables"], c["block_size"], c["seq_lens"])
        if c["out"].dtype == torch.float32:
            torch.testing.assert_close(out, c["out"], atol=1e-5, rtol=1e-5, msg=c["name"])
        else:
            # the reference's fp32 result, rounded to nearest even as the GPU stores it
            assert_close(out, c["out_f32"].to(c["out"].dtype), c["name"], min_exact=0.99)
            out32 = oracle.paged_attention_decode(
                c["query"].float(), c["k_cache"].float(), c["v_cache"].float(),
                c["block_tables"], c["block_size"], c["seq_lens"])
            torch.testing.assert_close(out32, c["out_f32"], atol=1e-5, rtol=1e-5, msg=c["name"])
        assert torch.isfinite(out).all(), c["name"]


def test_varlen_attention_matches_reference_kernel():
    """The oracle against the reference's own Triton prefill attention, run
    under Triton's interpreter, in fp32 (see make_golden.py for why bf16 is
    not in the fixture)."""
    g = load_golden("varlen_attention.pt")
    for c in g["cases"]:
        out = oracle.varlen_attention(c["q"], c["k"], c["v"], c["cu_seqlens"], c["cu_seqlens"],
                                      c["causal"])
        torch.testing.assert_close(out, c["out"], atol=1e-5, rtol=1e-5, msg=c["name"])


def test_sampler_matches_reference():
    """The oracle's sampler against the reference's sample_tokens on every
    fixture row: the same algorithm in torch on the CPU, so the tokens agree
    exactly."""
    g = load_golden("sampling.pt")
    for c in g["cases"]:
        out = oracle.sample_tokens(c["logits"], c["temperature"], c["top_k"], c["top_p"],
                                   c["uniforms"])
        assert out.dtype == torch.int64
        assert out.tolist() == c["out"].tolist(), c["name"]


def test_sampler_float64_decisions_agree_away_from_boundaries():
    """The float64 restatement (used to tell which rows sit on a decision
    boundary) picks the reference's token on every row whose margin exceeds
    the reference's own float32 rounding (its softmax sum's distance from 1,
    plus the cumsum rounding)."""
    g = load_golden("sampling.pt")
    for c in g["cases"]:
        toks, margins, slack = oracle.sample_margins(c["logits"], c["temperature"], c["top_k"],
                                                     c["top_p"], c["uniforms"])
        clear = margins > slack
        assert clear.float().mean() > 0.75, c["name"]
        assert toks[clear].tolist() == c["out"][clear].tolist(), c["name"]


def test_counter_hash_matches_reference():
    h = load_golden("sampling.pt")["hash"]
    for sd, st, m, u in zip(h["seeds"], h["steps"], h["mix64"], h["uniform"]):
        assert oracle.mix64(sd, st) == m
        assert oracle.uniform_from_hash(sd, st) == u
        assert 0.0 <= u < 1.0
    assert torch.equal(oracle.uniforms_from_seeds(h["seeds"], h["steps"]), h["uniforms_f32"])
