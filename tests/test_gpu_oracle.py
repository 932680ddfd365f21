"""CUDA path vs the CPU oracle on the benchmark configurations' seeded batches.

Every op of the path runs on the GPU through the C ABI and on the CPU oracle
(pinned to the reference by tests/test_oracle_golden.py) on the same inputs:
c1 and c3 in full, c2/c4/c5 on a token prefix the oracle finishes in seconds
(c5 with a cache whose element offsets exceed 2^31, so int64 addressing is on
the path).  Full-size batches are covered by tests/test_gpu_properties.py.
"""

import pytest
import torch

import tinyserver_b200 as tsb
from oracle import oracle
from tests.common import assert_close, assert_untouched, snapshot_pool
from tinyserver_b200 import workloads as W

pytestmark = pytest.mark.gpu

CASES = {
    # name: (max_tokens, num_blocks)
    "c1": (None, None),
    "c2": (3072, None),
    "c3": (None, None),
    "c4": (8192, None),
    "c5": (2048, 270_000),
}


@pytest.fixture(autouse=True)
def _no_device_flags():
    yield
    tsb.check_errors()


@pytest.fixture(scope="module", params=list(CASES))
def batch(request):
    max_tokens, nblk = CASES[request.param]
    b = W.make_batch(request.param, "cuda", max_tokens=max_tokens, num_blocks=nblk)
    yield b
    del b.tensors
    torch.cuda.empty_cache()


def test_embedding(batch):
    t = batch.tensors
    out = tsb.embedding(t["input_ids"], t["embed_weight"])
    ids = t["input_ids"].cpu()
    rows = t["embed_weight"][t["input_ids"]].cpu()  # only the gathered rows leave the GPU
    uniq, inv = torch.unique(ids, return_inverse=True)
    table = t["embed_weight"][uniq.cuda()].cpu()
    ref = oracle.embedding(inv, table)
    assert torch.equal(ref, rows)
    assert torch.equal(out.cpu(), ref)


def test_add_rmsnorm_both_norms(batch):
    t, s = batch.tensors, batch.cfg.shape
    y1, h1 = tsb.fused_add_rms_norm(t["x_mlp"], t["residual"], t["input_layernorm"], s.eps)
    ry1, rh1 = oracle.add_rmsnorm(t["x_mlp"].cpu(), t["residual"].cpu(),
                                  t["input_layernorm"].cpu(), s.eps)
    assert torch.equal(h1.cpu(), rh1)
    assert_close(y1, ry1, "input_layernorm", min_exact=0.99)
    y2, h2 = tsb.fused_add_rms_norm(t["attn_out"], h1, t["post_attention_layernorm"], s.eps)
    ry2, rh2 = oracle.add_rmsnorm(t["attn_out"].cpu(), rh1, t["post_attention_layernorm"].cpu(),
                                  s.eps)
    assert torch.equal(h2.cpu(), rh2)
    assert_close(y2, ry2, "post_attention_layernorm", min_exact=0.99)


def test_plain_rmsnorm(batch):
    t, s = batch.tensors, batch.cfg.shape
    y = tsb.rms_norm(t["residual"], t["input_layernorm"], s.eps)
    assert_close(y, oracle.rmsnorm(t["residual"].cpu(), t["input_layernorm"].cpu(), s.eps),
                 "rmsnorm", min_exact=0.99)


def test_rope_cos_sin(batch):
    t, s = batch.tensors, batch.cfg.shape
    cos, sin = tsb.rope_cos_sin(t["positions"], t["inv_freq"], s.head_dim, batch.cfg.dtype)
    rc, rs = oracle.rope_cos_sin(t["positions"].cpu(), t["inv_freq"].cpu(), s.head_dim,
                                 batch.cfg.dtype)
    assert_close(cos, rc, "cos", min_exact=0.99)
    assert_close(sin, rs, "sin", min_exact=0.99)


@pytest.mark.parametrize("cos_mode", ["table", "computed"])
def test_qk_norm_rope_store(batch, cos_mode):
    t, s = batch.tensors, batch.cfg.shape
    q, k, v = W.qkv_views(t["qkv"], s)
    cos, sin = tsb.rope_cos_sin(t["positions"], t["inv_freq"], s.head_dim, batch.cfg.dtype)
    pool = t["kv_pool"]
    bm, sm = t["block_mapping"], t["slot_mapping"]
    before_rows = pool[:, 0, bm, :, sm, :].clone()
    snap = snapshot_pool(pool)
    kw = dict(positions=t["positions"], inv_freq=t["inv_freq"]) if cos_mode == "computed" else {}
    q_out, k_out = tsb.qk_norm_rope_store(
        q, k, v, t["q_norm"], t["k_norm"], s.eps,
        cos if cos_mode == "table" else None, sin if cos_mode == "table" else None,
        t["k_cache"], t["v_cache"], bm, sm, **kw)
    rq, rk = oracle.qk_norm_rope_store(q.cpu(), k.cpu(), None, t["q_norm"].cpu(),
                                       t["k_norm"].cpu(), s.eps, cos.cpu(), sin.cpu())
    assert_close(q_out, rq, "q_out", min_exact=0.99)
    assert_close(k_out, rk, "k_out", min_exact=0.99)
    rows = pool[:, 0, bm, :, sm, :]  # (T, 2, Hkv, D)
    assert torch.equal(rows[:, 0], k_out), "K pages != rotated K"
    assert torch.equal(rows[:, 1], v), "V pages != V"
    assert_untouched(pool, snap, bm, sm)
    del snap
    pool[:, 0, bm, :, sm, :] = before_rows  # leave the cache as the batch made it


def test_store_kv_cache_batched_full_batch(batch):
    t, s = batch.tensors, batch.cfg.shape
    _, k, v = W.qkv_views(t["qkv"], s)
    k_src, v_src = k.transpose(0, 1), v.transpose(0, 1)  # (Hkv, T, D) strided views
    pool = t["kv_pool"]
    bm32 = t["block_mapping"].to(torch.int32)
    sm32 = t["slot_mapping"].to(torch.int32)
    tsb.store_kv_cache_batched(k_src, v_src, t["k_cache"], t["v_cache"], bm32, sm32)
    rows = pool[:, 0, t["block_mapping"], :, t["slot_mapping"], :]
    assert torch.equal(rows[:, 0], k) and torch.equal(rows[:, 1], v)


def test_store_kv_cache_per_sequence_matches_batched(batch):
    t, s = batch.tensors, batch.cfg.shape
    _, k, v = W.qkv_views(t["qkv"], s)
    pool = t["kv_pool"]
    tsb.store_kv_cache_batched(k.transpose(0, 1), v.transpose(0, 1), t["k_cache"], t["v_cache"],
                               t["block_mapping"], t["slot_mapping"])
    snap = pool[:, 0, t["block_mapping"], :, t["slot_mapping"], :].clone()
    pool[:, 0, t["block_mapping"], :, t["slot_mapping"], :] = 0
    cu_ = batch.cu_seqlens.tolist()
    for si, (n, p0) in enumerate(batch.seqs[:64]):  # per-sequence launches: first 64 seqs
        lo, hi = cu_[si], cu_[si + 1]
        tsb.store_kv_cache(p0, t["block_tables"][si], k[lo:hi].transpose(0, 1),
                           v[lo:hi].transpose(0, 1), t["k_cache"], t["v_cache"])
    upto = cu_[min(64, len(batch.seqs))]
    got = pool[:, 0, t["block_mapping"][:upto], :, t["slot_mapping"][:upto], :]
    assert torch.equal(got, snap[:upto])


def test_build_slot_mapping(batch):
    t = batch.tensors
    bm, sm = tsb.build_slot_mapping(t["cu_seqlens"], t["positions"], t["block_tables"],
                                    batch.cfg.block_size)
    assert torch.equal(bm, t["block_mapping"]) and torch.equal(sm, t["slot_mapping"])


def test_silu_and_mul(batch):
    t = batch.tensors
    I = batch.cfg.shape.intermediate
    out = tsb.silu_and_mul(t["gate_up"])
    g = t["gate_up"][:, :I].cpu()
    u = t["gate_up"][:, I:].cpu()
    assert_close(out, oracle.silu_and_mul(g, u), "silu_and_mul", min_exact=0.99)
