"""Generate the golden fixtures in tests/golden/ from the reference's own code.

Run in a container that has the reference checkout, named by ``--ref`` or
``TINYSERVER_REF`` (the script stops with a message when neither is given);
the GPU box never runs this script, it only reads the fixtures it wrote::

    python tests/golden/make_golden.py --ref /path/to/tinyserver

What produces the golden outputs:

* ``layer_{bf16,f32}.pt`` -- one forward of a 1-layer random-init Qwen3 model
  (transformers 5.5.0) patched by the reference's ``qwen3_model_patcher``
  (server/model/patches/qwen3.py:469-479), for a prefill batch and then a
  decode step, exactly as the reference's test helpers drive it
  (tests/model/paged_helpers.py:37-77).  Forward hooks capture every
  memory-bound op on the hot path: the embedding gather, input/post-attention
  RMSNorm with the residual add, q_norm/k_norm, the output of
  ``apply_rotary_pos_emb`` (wrapped where qwen3.py imports it), the paged KV
  cache before/after the reference's Triton store kernels, and the SiLU-and-mul
  product that feeds down_proj.  The Triton kernels run on CPU through Triton's
  interpreter (TRITON_INTERPRET=1).
* ``kv_store.pt`` -- the reference's two store kernels
  (server/model/kernels/kv_cache.py) on the scenarios of the reference's own
  tests (tests/model/test_kv_cache_kernels.py:73-207) plus a bf16, head_dim 128
  case with a permuted block table, int64 mappings and a poisoned cache.
* ``rope_cos_sin.pt`` -- Qwen3RotaryEmbedding (theta 1e6, head_dim 128) at
  positions up to 131071 in fp32 and bf16.
* ``outliers.pt`` -- Qwen3RMSNorm with the decoder layer's residual add at
  hidden 4096 with x50 outliers, and ACT2FN["silu"](gate) * up on
  large-magnitude inputs, in bf16.
* ``paged_attention.pt`` -- the reference's decode paged-attention Triton
  kernel (server/model/kernels/paged_attention.py) on its own tests'
  configurations plus bf16 GQA cases longer than one partition.
* ``varlen_attention.pt`` -- the reference's prefill varlen attention kernel
  (server/model/kernels/varlen_attention.py), causal and not, MHA and GQA,
  fp32 (the interpreter cannot run it in bf16).
* ``sampling.pt`` -- the reference's batched sampler and counter-based noise
  (server/model/sampling.py, server/model/determinism.py) on hand-checkable
  rows, Qwen3-vocabulary bf16 rows, tie-heavy fp32 rows and fp16 extremes.
"""

from __future__ import annotations

import argparse
import os
import sys

os.environ.setdefault("TRITON_INTERPRET", "1")

import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))


def _seeded_(module: torch.nn.Module, gen: torch.Generator) -> None:
    """Overwrite every parameter with seeded values: N(0, 0.02) for matrices,
    1 + N(0, 0.02) for norm weights (vectors)."""
    with torch.no_grad():
        for name, p in module.named_parameters():
            noise = torch.randn(p.shape, generator=gen, dtype=torch.float32) * 0.02
            if p.dim() == 1:
                p.copy_(1.0 + noise)
            else:
                p.copy_(noise)


def _layer_case(dtype: torch.dtype, seq_lens: list[int], seed: int, vocab: int,
                num_blocks: int) -> dict:
    from transformers import Qwen3Config, Qwen3ForCausalLM

    import server.model.patches.qwen3 as refq
    from server.model.inference_context import InferenceContext, inference_context
    from server.model.prefill_helpers import build_prefill_inputs

    gen = torch.Generator().manual_seed(seed)
    cfg = Qwen3Config(
        vocab_size=vocab, hidden_size=1024, intermediate_size=1024, num_hidden_layers=1,
        num_attention_heads=16, num_key_value_heads=8, head_dim=128, rms_norm_eps=1e-6,
        rope_parameters={"rope_type": "default", "rope_theta": 1e6},
        max_position_embeddings=40960, tie_word_embeddings=False,
    )
    model = Qwen3ForCausalLM(cfg).eval()
    _seeded_(model, gen)
    model = model.to(dtype)
    layer = model.model.layers[0]
    attn = layer.self_attn

    block_size = 16
    pool = torch.randn(2, 1, num_blocks, 8, block_size, 128, generator=gen).to(dtype)
    refq.qwen3_model_patcher(model)
    attn.k_cache = pool[0, 0]
    attn.v_cache = pool[1, 0]

    cap: dict[str, list] = {}

    def hook(name):
        def fn(_mod, args, out):
            cap.setdefault(name + ".in", []).append(args[0].detach().clone())
            o = out[0] if isinstance(out, tuple) else out
            cap.setdefault(name + ".out", []).append(o.detach().clone())
        return fn

    model.model.embed_tokens.register_forward_hook(hook("embed"))
    layer.input_layernorm.register_forward_hook(hook("input_layernorm"))
    layer.post_attention_layernorm.register_forward_hook(hook("post_attention_layernorm"))
    attn.q_proj.register_forward_hook(hook("q_proj"))
    attn.k_proj.register_forward_hook(hook("k_proj"))
    attn.v_proj.register_forward_hook(hook("v_proj"))
    attn.q_norm.register_forward_hook(hook("q_norm"))
    attn.k_norm.register_forward_hook(hook("k_norm"))
    attn.o_proj.register_forward_hook(hook("o_proj"))
    layer.mlp.gate_proj.register_forward_hook(hook("gate_proj"))
    layer.mlp.up_proj.register_forward_hook(hook("up_proj"))
    layer.mlp.down_proj.register_forward_hook(hook("down_proj"))
    # inputs that repeat another capture (every projection reads the normed
    # hidden state; q/k_norm read the projections; rope reads q/k_norm's output)
    redundant = {"q_proj.in", "k_proj.in", "v_proj.in", "gate_proj.in", "up_proj.in",
                 "q_norm.in", "k_norm.in", "o_proj.in", "post_attention_layernorm.out.dup"}

    orig_rope = refq.apply_rotary_pos_emb

    def rope_wrap(q, k, cos, sin, *a, **kw):
        qo, ko = orig_rope(q, k, cos, sin, *a, **kw)
        cap.setdefault("rope.cos", []).append(cos.detach().clone())
        cap.setdefault("rope.sin", []).append(sin.detach().clone())
        cap.setdefault("rope.q_out", []).append(qo.detach().clone())
        cap.setdefault("rope.k_out", []).append(ko.detach().clone())
        return qo, ko

    refq.apply_rotary_pos_emb = rope_wrap

    perm = torch.randperm(num_blocks, generator=gen).tolist()
    # capacity for prompt + one decode token per sequence
    need = [-(-(n + 1) // block_size) for n in seq_lens]
    block_tables, cur = [], 0
    for n in need:
        block_tables.append(perm[cur:cur + n])
        cur += n
    assert cur <= num_blocks
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=gen).tolist() for n in seq_lens]

    cache_before = pool.clone()
    written_prefill = [(bt[j // block_size], j % block_size)
                       for n, bt in zip(seq_lens, block_tables) for j in range(n)]
    written_decode = [(bt[n // block_size], n % block_size)
                      for n, bt in zip(seq_lens, block_tables)]
    input_ids, position_ids, ctx = build_prefill_inputs(prompts, block_tables, "cpu")
    try:
        with torch.no_grad(), inference_context(ctx):
            model(input_ids=input_ids, position_ids=position_ids, use_cache=False)
        cache_after_prefill = pool.clone()
        next_tokens = torch.randint(0, cfg.vocab_size, (len(seq_lens),), generator=gen).tolist()
        dec_ids = torch.tensor([next_tokens], dtype=torch.long)
        dec_pos = torch.tensor([seq_lens], dtype=torch.long)
        dctx = InferenceContext(mode="decode", sequences=[
            {"num_tokens": 1, "block_table": bt} for bt in block_tables])
        with torch.no_grad(), inference_context(dctx):
            model(input_ids=dec_ids, position_ids=dec_pos, use_cache=False)
        cache_after_decode = pool.clone()
    finally:
        refq.apply_rotary_pos_emb = orig_rope

    out = {
        "dtype": str(dtype), "hidden": 1024, "num_q_heads": 16, "num_kv_heads": 8,
        "head_dim": 128, "intermediate": 1024, "eps": 1e-6, "rope_theta": 1e6,
        "block_size": block_size, "num_blocks": num_blocks, "seq_lens": seq_lens,
        "block_tables": block_tables, "prefill_input_ids": input_ids.clone(),
        "prefill_position_ids": position_ids.clone(), "decode_input_ids": dec_ids,
        "decode_position_ids": dec_pos, "embed_weight": model.model.embed_tokens.weight.detach().clone(),
        "input_layernorm_weight": layer.input_layernorm.weight.detach().clone(),
        "post_attention_layernorm_weight": layer.post_attention_layernorm.weight.detach().clone(),
        "q_norm_weight": attn.q_norm.weight.detach().clone(),
        "k_norm_weight": attn.k_norm.weight.detach().clone(),
        "inv_freq": model.model.rotary_emb.inv_freq.detach().clone(),
        "cache_before": cache_before,
        "written_prefill": written_prefill, "written_decode": written_decode,
        "rows_after_prefill": _written_rows(cache_before, cache_after_prefill, written_prefill),
        "rows_after_decode": _written_rows(cache_after_prefill, cache_after_decode,
                                           written_decode),
    }
    for key, vals in cap.items():
        if key in redundant:
            continue
        assert len(vals) == 2, (key, len(vals))  # [prefill, decode]
        out[key] = vals
    return out


def _written_rows(before: torch.Tensor, after: torch.Tensor, written: list) -> torch.Tensor:
    """Rows (2, len(written), Hkv, D) of the (K, V) pool at the written (block, slot)
    pairs, after checking that no other cache row changed.  before/after are
    pools of shape (2, 1, N, Hkv, B, D)."""
    changed = after.ne(before).any(dim=-1)  # (2, 1, N, Hkv, B)
    expect = torch.zeros_like(changed)
    for b, s in written:
        expect[:, :, b, :, s] = True
    assert not (changed & ~expect).any(), "reference wrote outside the mapped slots"
    idx_b = torch.tensor([b for b, _ in written])
    idx_s = torch.tensor([s for _, s in written])
    return after[:, 0, idx_b, :, idx_s, :].clone()


def _kv_store_case() -> dict:
    from server.model.kernels.kv_cache import store_kv_cache, store_kv_cache_batched

    gen = torch.Generator().manual_seed(4321)
    cases = []
    # The scenarios of tests/model/test_kv_cache_kernels.py:73-207 (fp32).
    scen = [
        ("single_seq", 2, 4, 8, 2, [{"start_pos": 0, "seq_len": 4, "block_table": [0]}]),
        ("multiple_seqs", 4, 4, 16, 4, [
            {"start_pos": 0, "seq_len": 3, "block_table": [0]},
            {"start_pos": 0, "seq_len": 5, "block_table": [1, 2]},
            {"start_pos": 0, "seq_len": 4, "block_table": [3]}]),
        ("multi_block", 2, 4, 32, 3, [{"start_pos": 0, "seq_len": 12, "block_table": [0, 1, 2]}]),
        ("single_token", 2, 4, 8, 3, [
            {"start_pos": 0, "seq_len": 1, "block_table": [0]},
            {"start_pos": 0, "seq_len": 1, "block_table": [1]},
            {"start_pos": 0, "seq_len": 1, "block_table": [2]}]),
        ("nonzero_start", 2, 4, 8, 3, [
            {"start_pos": 4, "seq_len": 3, "block_table": [0, 1]},
            {"start_pos": 8, "seq_len": 4, "block_table": [0, 0, 2]}]),
    ]
    for name, hkv, bsz, hd, nblk, seqs in scen:
        cases.append(_store_one(name, torch.float32, hkv, bsz, hd, nblk, seqs, torch.int32, gen,
                                store_kv_cache, store_kv_cache_batched, poison=False))
    # bf16, Qwen3 head geometry, permuted blocks, int64 mappings, poisoned cache.
    perm = torch.randperm(16, generator=gen).tolist()
    seqs = [
        {"start_pos": 0, "seq_len": 37, "block_table": perm[0:3]},
        {"start_pos": 21, "seq_len": 20, "block_table": perm[3:6]},
        {"start_pos": 0, "seq_len": 1, "block_table": perm[6:7]},
        {"start_pos": 95, "seq_len": 1, "block_table": perm[7:14]},
    ]
    cases.append(_store_one("bf16_permuted", torch.bfloat16, 8, 16, 128, 16, seqs, torch.int64,
                            gen, store_kv_cache, store_kv_cache_batched, poison=True))
    return {"cases": cases}


def _store_one(name, dtype, hkv, bsz, hd, nblk, seqs, idx_dtype, gen, per_seq, batched, poison):
    k_srcs = [torch.randn(hkv, s["seq_len"], hd, generator=gen).to(dtype) for s in seqs]
    v_srcs = [torch.randn(hkv, s["seq_len"], hd, generator=gen).to(dtype) for s in seqs]
    shape = (nblk, hkv, bsz, hd)
    if poison:
        base_k = torch.randn(shape, generator=gen).to(dtype)
        base_v = torch.randn(shape, generator=gen).to(dtype)
    else:
        base_k = torch.zeros(shape, dtype=dtype)
        base_v = torch.zeros(shape, dtype=dtype)
    # per-sequence kernel (kv_cache.py:6-119)
    k_ref, v_ref = base_k.clone(), base_v.clone()
    for s, ks, vs in zip(seqs, k_srcs, v_srcs):
        per_seq(s["start_pos"], torch.tensor(s["block_table"], dtype=torch.int32), ks, vs,
                k_ref, v_ref)
    # batched kernel (kv_cache.py:122-251) with the reference tests' mapping recipe
    # (tests/model/test_kv_cache_kernels.py:16-37)
    bm, sm = [], []
    for s in seqs:
        for i in range(s["seq_len"]):
            p = s["start_pos"] + i
            bm.append(s["block_table"][p // bsz])
            sm.append(p % bsz)
    bm_t = torch.tensor(bm, dtype=idx_dtype)
    sm_t = torch.tensor(sm, dtype=idx_dtype)
    k_bat, v_bat = base_k.clone(), base_v.clone()
    batched(torch.cat(k_srcs, 1), torch.cat(v_srcs, 1), k_bat, v_bat, bm_t, sm_t)
    assert torch.equal(k_bat, k_ref) and torch.equal(v_bat, v_ref), name
    assert len(set(zip(bm, sm))) == len(bm), "golden mappings must not collide"
    pool_before = torch.stack([base_k, base_v])[:, None]
    pool_after = torch.stack([k_bat, v_bat])[:, None]
    return {"name": name, "seqs": seqs, "k_srcs": k_srcs, "v_srcs": v_srcs,
            "cache_k_before": base_k, "cache_v_before": base_v,
            "block_mapping": bm_t, "slot_mapping": sm_t,
            "written_rows": _written_rows(pool_before, pool_after, list(zip(bm, sm)))}


def _rope_case() -> dict:
    from transformers import Qwen3Config
    from transformers.models.qwen3.modeling_qwen3 import Qwen3RotaryEmbedding

    cfg = Qwen3Config(hidden_size=1024, num_attention_heads=16, num_key_value_heads=8,
                      head_dim=128, rope_parameters={"rope_type": "default", "rope_theta": 1e6},
                      max_position_embeddings=131072)
    rot = Qwen3RotaryEmbedding(cfg)
    gen = torch.Generator().manual_seed(77)
    pos = torch.cat([torch.arange(0, 64), torch.randint(0, 131072, (192,), generator=gen),
                     torch.tensor([8191, 16383, 32767, 65535, 131071])]).to(torch.int64)[None]
    out = {"positions": pos, "inv_freq": rot.inv_freq.clone(), "head_dim": 128,
           "rope_theta": 1e6}
    for dt in (torch.float32, torch.bfloat16):
        cos, sin = rot(torch.zeros(1, dtype=dt), pos)
        out[f"cos_{dt}"] = cos[0]
        out[f"sin_{dt}"] = sin[0]
    return out


def _outlier_case() -> dict:
    from transformers.activations import ACT2FN
    from transformers.models.qwen3.modeling_qwen3 import Qwen3RMSNorm

    gen = torch.Generator().manual_seed(99)
    H, T = 4096, 24
    x = torch.randn(T, H, generator=gen)
    mask = torch.rand(T, H, generator=gen) < 0.001
    x = torch.where(mask, x * 50.0, x).to(torch.bfloat16)
    res = torch.randn(T, H, generator=gen).mul(0.5).to(torch.bfloat16)
    norm = Qwen3RMSNorm(H, eps=1e-6)
    with torch.no_grad():
        norm.weight.copy_(1.0 + 0.02 * torch.randn(H, generator=gen))
    norm = norm.to(torch.bfloat16)
    with torch.no_grad():
        h = res + x  # Qwen3DecoderLayer residual add (HF:327)
        y = norm(h)
    I = 2048
    gate = (torch.randn(T, I, generator=gen) * 6.0).to(torch.bfloat16)
    gate[0, :8] = torch.tensor([-100., -50., -20., -1e-3, 0., 1e-3, 20., 90.])
    up = torch.randn(T, I, generator=gen).to(torch.bfloat16)
    with torch.no_grad():
        act = ACT2FN["silu"](gate) * up  # Qwen3MLP (HF:82)
    return {"x": x, "residual": res, "weight": norm.weight.detach().clone(), "eps": 1e-6,
            "h": h, "y": y, "gate": gate, "up": up, "act": act}


def _paged_attention_case() -> dict:
    """The reference's decode paged-attention Triton kernel
    (server/model/kernels/paged_attention.py:124-192) under Triton's
    interpreter on: the three configurations of its own tests
    (tests/model/test_paged_attention_kernel.py:109-116) in fp32, its poisoned
    partial-block case (:180-214), and bf16 GQA cases with sequences longer
    than one 512-key partition (group sizes 4 and 8)."""
    from server.model.kernels.paged_attention import paged_attention_forward

    gen = torch.Generator().manual_seed(2024)
    cases = []
    for name, hq, hkv, hd, bsz, lens, dt, poison in (
            ("mha-single-block", 4, 4, 64, 16, [10], torch.float32, False),
            ("gqa-ragged", 8, 2, 64, 16, [7, 16, 40], torch.float32, False),
            ("gqa-headdim128", 16, 4, 128, 32, [1, 33, 64], torch.float32, False),
            ("partial-block-poisoned", 8, 2, 64, 16, [5], torch.float32, True),
            ("bf16-g4-split", 8, 2, 128, 16, [1, 15, 17, 300, 700], torch.bfloat16, False),
            ("bf16-g8-split", 16, 2, 128, 16, [33, 600], torch.bfloat16, False)):
        per = [max(1, -(-n // bsz)) for n in lens]
        nblk = sum(per) + 3
        q = torch.randn(len(lens), hq, hd, generator=gen).to(dt)
        kc = torch.randn(nblk, hkv, bsz, hd, generator=gen).to(dt)
        vc = torch.randn(nblk, hkv, bsz, hd, generator=gen).to(dt)
        phys = torch.randperm(nblk, generator=gen)[:sum(per)]
        bt = torch.zeros(len(lens), max(per), dtype=torch.int32)
        cur = 0
        for i, n in enumerate(per):
            bt[i, :n] = phys[cur:cur + n].to(torch.int32)
            cur += n
        if poison:
            blk = int(bt[0, 0])
            kc[blk, :, lens[0]:, :] = 1e4
            vc[blk, :, lens[0]:, :] = 1e4
        sl = torch.tensor(lens, dtype=torch.int32)
        out = paged_attention_forward(q, kc, vc, bt, bsz, sl)
        case = {"name": name, "query": q, "k_cache": kc, "v_cache": vc, "block_tables": bt,
                "block_size": bsz, "seq_lens": sl, "out": out}
        if dt != torch.float32:
            # The kernel upcasts its loads to fp32 (paged_attention.py:72, :90-95), so the
            # same kernel on fp32 copies of the inputs gives its exact fp32 result before
            # the final store.  Triton's interpreter stores fp32 into a bf16 tensor by
            # truncation, while the GPU rounds to nearest even; the expected bf16 output
            # is out_f32 rounded to nearest even.
            case["out_f32"] = paged_attention_forward(q.float(), kc.float(), vc.float(), bt,
                                                      bsz, sl)
        cases.append(case)
    return {"cases": cases}


def _varlen_attention_case() -> dict:
    """The reference's prefill varlen attention Triton kernel
    (server/model/kernels/varlen_attention.py:145-218) under Triton's
    interpreter: causal and non-causal, MHA and GQA, ragged packed lengths,
    fp32 only.  Triton's interpreter cannot run this kernel in bf16 (its
    bf16 tl.dot returned values of order 1e8 for unit-variance inputs), so
    the bf16 rounding points -- p cast to the value dtype (:121), the final
    store -- are restated in the oracle from the source and the fp32 cases
    pin everything else."""
    from server.model.kernels.varlen_attention import flash_attn_varlen_func

    gen = torch.Generator().manual_seed(4242)
    cases = []
    for name, lens, hq, hkv, hd, causal, dt in (
            ("mha-causal-d64", [5, 3, 7], 4, 4, 64, True, torch.float32),
            ("gqa-causal-ragged", [1, 33, 64, 100], 8, 2, 128, True, torch.float32),
            ("mha-noncausal", [17, 40], 8, 8, 128, False, torch.float32),
            ("c1-lengths", [37, 64, 128, 255], 4, 2, 64, True, torch.float32)):
        T = sum(lens)
        q = torch.randn(T, hq, hd, generator=gen).to(dt)
        k = torch.randn(T, hkv, hd, generator=gen).to(dt)
        v = torch.randn(T, hkv, hd, generator=gen).to(dt)
        cu = torch.zeros(len(lens) + 1, dtype=torch.int32)
        cu[1:] = torch.cumsum(torch.tensor(lens), 0)
        out = flash_attn_varlen_func(q, k, v, cu, cu, max(lens), max(lens), causal=causal)
        cases.append({"name": name, "q": q, "k": k, "v": v, "cu_seqlens": cu,
                      "max_seqlen": max(lens), "causal": causal, "out": out})
    return {"cases": cases}


def _sampling_case() -> dict:
    """The reference's batched sampler (server/model/sampling.py:118-194) and
    its counter-based noise (server/model/determinism.py:30-73), run as
    shipped on the CPU:

    * small hand-checkable rows in the spirit of the reference's own tests
      (tests/model/test_batch_sampling.py): equal logits, a greedy tie, per-row
      top-k 1/2/3, a tiny top-p, top-k above the vocabulary, u = 0 and u near 1;
    * bf16 rows at Qwen3's vocabulary (151936) with mixed temperature / top-k /
      top-p and uniforms from the hash;
    * fp32 integer-valued logits (long runs of equal values, where the stable
      sort's index order decides) with -inf entries;
    * fp16 rows with top_p 0, top_k 1, extreme temperatures;
    * uniform_from_hash at edge seeds and steps.
    """
    from server.model.determinism import mix64, uniform_from_hash, uniforms_from_seeds
    from server.model.sampling import sample_tokens

    gen = torch.Generator().manual_seed(77)
    cases = []

    def add(name, logits, temperature, top_k, top_p, uniforms):
        out = sample_tokens(logits, temperature, top_k, top_p, uniforms)
        cases.append({"name": name, "logits": logits, "temperature": temperature,
                      "top_k": top_k, "top_p": top_p, "uniforms": uniforms, "out": out})

    f32, i64 = torch.float32, torch.int64
    row = [5.0, 4.0, 3.0, 2.0, 1.0, 0.0]
    small = torch.tensor([[0.0, 0.0, 0.0, 0.0, 0.0, 0.0]] * 4 + [[0.0, 5.0, 5.0, 1.0, 0.0, 0.0]]
                         + [row] * 3 + [[-10.0, -10.0, 10.0, -10.0, -10.0, -10.0]] * 2
                         + [[1.0, 9.0, 3.0, 7.0, 2.0, 0.5]] * 2, dtype=f32)
    add("hand", small,
        torch.tensor([1.0] * 4 + [0.0] + [1.0] * 7, dtype=f32),
        torch.tensor([0] * 5 + [1, 2, 3] + [0, 999, 0, 0], dtype=i64),
        torch.tensor([1.0] * 8 + [1e-6, 1.0, 1.0, 0.5], dtype=f32),
        torch.tensor([0.1, 0.4, 0.6, 0.9, 0.99, 0.999, 0.999, 0.999, 0.9, 0.3, 0.0,
                      1.0 - 2.0 ** -24], dtype=f32))

    B, V = 8, 151936
    logits = (torch.randn(B, V, generator=gen) * 3.0).to(torch.bfloat16)
    add("bf16-qwen3-vocab", logits,
        torch.tensor([0.0, 0.6, 0.8, 1.0, 1.0, 0.7, 1.2, 0.9], dtype=f32),
        torch.tensor([0, 0, 50, 0, 20, 1000, 0, 40], dtype=i64),
        torch.tensor([1.0, 0.9, 0.95, 1.0, 0.8, 0.9, 0.6, 1.0], dtype=f32),
        uniforms_from_seeds(list(range(100, 100 + B)), [7] * B))

    B, V = 64, 4096
    logits = torch.randint(-8, 9, (B, V), generator=gen).to(f32)
    logits[::5, ::7] = float("-inf")
    add("f32-ties", logits,
        torch.tensor([0.5, 1.0, 2.0, 0.0] * 16, dtype=f32),
        torch.tensor([0, 7, 100, 0, 4095, 4096, 1, 300] * 8, dtype=i64),
        torch.tensor([1.0, 0.9, 0.3, 0.99, 0.5, 1.0, 0.7, 0.05] * 8, dtype=f32),
        uniforms_from_seeds([s * 7919 for s in range(B)], list(range(B))))

    B, V = 16, 32000
    logits = (torch.randn(B, V, generator=gen) * 2.0).to(torch.float16)
    add("f16-extremes", logits,
        torch.tensor([1e-6, 50.0, 1.0, 1.0] * 4, dtype=f32),
        torch.tensor([0, 0, 1, 5] * 4, dtype=i64),
        torch.tensor([0.9, 0.95, 1.0, 0.0] * 4, dtype=f32),
        uniforms_from_seeds([2 ** 64 - 1 - s for s in range(B)], [10 ** 6] * B))

    seeds = [0, 1, 2, 42, 1234, 2 ** 31, 2 ** 63, 2 ** 64 - 1]
    steps = [0, 1, 9, 10_000, 2 ** 40]
    pairs = [(sd, st) for sd in seeds for st in steps]
    hash_case = {"seeds": [p[0] for p in pairs], "steps": [p[1] for p in pairs],
                 "mix64": [mix64(*p) for p in pairs],
                 "uniform": [uniform_from_hash(*p) for p in pairs],
                 "uniforms_f32": uniforms_from_seeds([p[0] for p in pairs],
                                                     [p[1] for p in pairs])}
    return {"cases": cases, "hash": hash_case}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("TINYSERVER_REF"),
                    help="the reference checkout (default: $TINYSERVER_REF)")
    ap.add_argument("--only", default=None, help="write just this fixture (e.g. paged_attention)")
    args = ap.parse_args()
    if not args.ref or not os.path.isdir(os.path.join(args.ref, "server", "model")):
        ap.error("give the reference checkout with --ref or TINYSERVER_REF (a directory that "
                 "holds server/model)")
    sys.path.insert(0, args.ref)
    import transformers
    torch.manual_seed(0)
    meta = {"transformers": transformers.__version__, "torch": torch.__version__}
    if args.only == "paged_attention":
        torch.save({**_paged_attention_case(), "meta": meta},
                   os.path.join(HERE, "paged_attention.pt"))
        return
    if args.only == "sampling":
        torch.save({**_sampling_case(), "meta": meta}, os.path.join(HERE, "sampling.pt"))
        return
    if args.only == "varlen_attention":
        torch.save({**_varlen_attention_case(), "meta": meta},
                   os.path.join(HERE, "varlen_attention.pt"))
        return
    for dt, lens, seed, vocab, nblk, fname in (
            (torch.bfloat16, [5, 16, 37], 1234, 128, 8, "layer_bf16.pt"),
            (torch.float32, [3, 17], 1235, 128, 4, "layer_f32.pt")):
        d = _layer_case(dt, lens, seed, vocab, nblk)
        d["meta"] = meta
        torch.save(d, os.path.join(HERE, fname))
    torch.save({**_kv_store_case(), "meta": meta}, os.path.join(HERE, "kv_store.pt"))
    torch.save({**_rope_case(), "meta": meta}, os.path.join(HERE, "rope_cos_sin.pt"))
    torch.save({**_outlier_case(), "meta": meta}, os.path.join(HERE, "outliers.pt"))
    torch.save({**_paged_attention_case(), "meta": meta}, os.path.join(HERE, "paged_attention.pt"))
    torch.save({**_varlen_attention_case(), "meta": meta},
               os.path.join(HERE, "varlen_attention.pt"))
    torch.save({**_sampling_case(), "meta": meta}, os.path.join(HERE, "sampling.pt"))
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".pt"):
            print(f, os.path.getsize(os.path.join(HERE, f)))


if __name__ == "__main__":
    main()
