"""Decode paged attention on the GPU against the reference's own kernel
outputs (golden vectors) and the CPU oracle.

Tolerances: fp32 |a - e| <= 1e-4 + 1e-4 |e| (the reference's own test uses
1e-3; the kernel's fast exp and summation order move the last fp32 bits);
16-bit outputs: the bf16/fp16 contract of tests/common.py with >= 98% of the
elements bit-exact against the reference's fp32 result rounded to nearest.
"""

import pytest
import torch

import tinyserver_b200 as tsb
from oracle import oracle
from tests.common import assert_close, load_golden

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _check(out, expected, what, min_exact=0.98):
    if expected.dtype == torch.float32:
        torch.testing.assert_close(out.cpu(), expected, atol=1e-4, rtol=1e-4, msg=what)
    else:
        assert_close(out, expected, what, min_exact=min_exact)


def _to(c, key):
    return c[key].to(DEV)


@pytest.mark.parametrize("split", [True, False])
def test_reference_golden_cases(split):
    g = load_golden("paged_attention.pt")
    for c in g["cases"]:
        out = tsb.paged_attention_forward(_to(c, "query"), _to(c, "k_cache"), _to(c, "v_cache"),
                                          _to(c, "block_tables"), c["block_size"],
                                          _to(c, "seq_lens"), split=split)
        tsb.check_errors()
        assert out.shape == c["query"].shape and out.dtype == c["query"].dtype
        expected = c["out"] if c["out"].dtype == torch.float32 else \
            c["out_f32"].to(c["out"].dtype)
        _check(out, expected, f"{c['name']} split={split}")
        assert torch.isfinite(out).all()


def _paged_inputs(lens, hq, hkv, hd, bsz, dtype, seed, extra_blocks=5):
    g = torch.Generator().manual_seed(seed)
    per = [max(1, -(-n // bsz)) for n in lens]
    nblk = sum(per) + extra_blocks
    q = torch.randn(len(lens), hq, hd, generator=g).to(dtype)
    kc = torch.randn(nblk, hkv, bsz, hd, generator=g).to(dtype)
    vc = torch.randn(nblk, hkv, bsz, hd, generator=g).to(dtype)
    phys = torch.randperm(nblk, generator=g)[:sum(per)]
    bt = torch.zeros(len(lens), max(per) + 2, dtype=torch.int32)
    cur = 0
    for i, n in enumerate(per):
        bt[i, :n] = phys[cur:cur + n].to(torch.int32)
        cur += n
    return q, kc, vc, bt, torch.tensor(lens, dtype=torch.int32)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("hq,hkv", [(8, 8), (8, 4), (32, 8), (64, 8)])
@pytest.mark.parametrize("hd", [64, 128, 256])
def test_shapes_against_oracle(dtype, hq, hkv, hd):
    lens = [1, 2, 31, 32, 33, 511, 512, 513, 1300]
    q, kc, vc, bt, sl = _paged_inputs(lens, hq, hkv, hd, 16, dtype, seed=hq * 1000 + hd)
    expected = oracle.paged_attention_decode(q, kc, vc, bt, 16, sl)
    out = tsb.paged_attention_forward(q.to(DEV), kc.to(DEV), vc.to(DEV), bt.to(DEV), 16,
                                      sl.to(DEV))
    tsb.check_errors()
    _check(out, expected, f"{dtype} {hq}/{hkv} d{hd}")


def test_decode_batch_at_qwen3_8b_shapes():
    """A c3-like decode step (Qwen3-8B heads, 16-token pages) on a subset of
    sequences, with the reference's large default page size too."""
    g = torch.Generator().manual_seed(7)
    lens = torch.randint(1, 4096, (24,), generator=g).tolist()
    for bsz in (16, 256):
        q, kc, vc, bt, sl = _paged_inputs(lens, 32, 8, 128, bsz, torch.bfloat16, seed=bsz)
        expected = oracle.paged_attention_decode(q, kc, vc, bt, bsz, sl)
        out = tsb.paged_attention_forward(q.to(DEV), kc.to(DEV), vc.to(DEV), bt.to(DEV), bsz,
                                          sl.to(DEV))
        tsb.check_errors()
        _check(out, expected, f"8B decode, block {bsz}")


def test_strided_layer_view_of_the_pool_and_strided_query():
    """The cache as the reference allocates it (per-layer views of one
    6-D pool, qwen3.py:49-62) and q as a strided view."""
    lens = [40, 700]
    q, kc, vc, bt, sl = _paged_inputs(lens, 32, 8, 128, 16, torch.bfloat16, seed=3)
    pool = torch.zeros(2, 3, *kc.shape, dtype=kc.dtype)
    pool[0, 1], pool[1, 1] = kc, vc
    pool = pool.to(DEV)
    big_q = torch.zeros(len(lens), 32, 2 * 128, dtype=q.dtype)
    big_q[:, :, :128] = q
    qv = big_q.to(DEV)[:, :, :128]
    q_before = qv.clone()
    out = tsb.paged_attention_forward(qv, pool[0, 1], pool[1, 1], bt.to(DEV), 16, sl.to(DEV))
    tsb.check_errors()
    _check(out, oracle.paged_attention_decode(q, kc, vc, bt, 16, sl), "pool view")
    assert torch.equal(qv, q_before), "query was modified"


def test_partial_last_block_is_masked():
    lens = [5, 21]
    q, kc, vc, bt, sl = _paged_inputs(lens, 8, 2, 64, 16, torch.float32, seed=9)
    for s, n in enumerate(lens):
        last = int(bt[s, (n - 1) // 16])
        kc[last, :, n % 16:, :] = 1e4
        vc[last, :, n % 16:, :] = 1e4
    out = tsb.paged_attention_forward(q.to(DEV), kc.to(DEV), vc.to(DEV), bt.to(DEV), 16,
                                      sl.to(DEV))
    tsb.check_errors()
    assert torch.isfinite(out).all()
    _check(out, oracle.paged_attention_decode(q, kc, vc, bt, 16, sl), "partial block")


def test_block_outside_the_cache_is_flagged_not_read():
    q, kc, vc, bt, sl = _paged_inputs([40], 8, 2, 64, 16, torch.float32, seed=4)
    bt[0, 1] = kc.shape[0] + 1000  # second logical block points outside the cache
    tsb.paged_attention_forward(q.to(DEV), kc.to(DEV), vc.to(DEV), bt.to(DEV), 16, sl.to(DEV))
    with pytest.raises(IndexError, match="block index"):
        tsb.check_errors()


@pytest.mark.parametrize("split", [True, False])
@pytest.mark.parametrize("bsz", [8, 16, 32])
def test_16bit_pages_with_poisoned_tails(bsz, split):
    """The 16-bit kernel copies each 16-key tile with cp.async, keys past the
    sequence zero-filled, at block sizes below, equal to and above the tile.
    Slots past each sequence's end hold NaN: none may reach the output,
    through S or through P V."""
    lens = [1, 5, 16, 17, 40, 300, 1029, 2048, 3000]
    q, kc, vc, bt, sl = _paged_inputs(lens, 32, 8, 128, bsz, torch.bfloat16, seed=bsz + 77)
    for s, n in enumerate(lens):
        if n % bsz:
            last = int(bt[s, (n - 1) // bsz])
            kc[last, :, n % bsz:, :] = float("nan")
            vc[last, :, n % bsz:, :] = float("nan")
    expected = oracle.paged_attention_decode(q, kc, vc, bt, bsz, sl)
    out = tsb.paged_attention_forward(q.to(DEV), kc.to(DEV), vc.to(DEV), bt.to(DEV), bsz,
                                      sl.to(DEV), split=split)
    tsb.check_errors()
    assert torch.isfinite(out).all()
    _check(out, expected, f"block {bsz} split={split}")


def test_16bit_block_outside_the_cache_is_flagged_not_read():
    """A bad block index in the middle of a 16-bit sequence: flagged, its
    keys zero-filled and masked, the output finite."""
    q, kc, vc, bt, sl = _paged_inputs([200], 32, 8, 128, 16, torch.bfloat16, seed=5)
    bt[0, 3] = kc.shape[0] + 1000
    out = tsb.paged_attention_forward(q.to(DEV), kc.to(DEV), vc.to(DEV), bt.to(DEV), 16,
                                      sl.to(DEV))
    with pytest.raises(IndexError, match="block index"):
        tsb.check_errors()
    assert torch.isfinite(out).all()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("split", [True, False])
def test_length_beyond_the_block_table_is_cut_and_flagged(dtype, split):
    """A seq_len longer than its block-table row can describe is cut to the
    row (no read past the row, no partial past the workspace) and flagged;
    the output equals a call with the cut length."""
    lens = [40, 700, 90]
    q, kc, vc, bt, sl = _paged_inputs(lens, 8, 2, 128, 16, dtype, seed=12)
    cap = bt.shape[1] * 16
    long = sl.clone()
    long[1] = cap + 3000  # far past the row: would need more partitions than the workspace has
    cut = torch.minimum(long, torch.tensor(cap, dtype=torch.int32))
    args = (q.to(DEV), kc.to(DEV), vc.to(DEV), bt.to(DEV), 16)
    tsb.check_errors()
    out = tsb.paged_attention_forward(*args, long.to(DEV), split=split)
    with pytest.raises(IndexError, match="beyond the block table"):
        tsb.check_errors()
    expected = tsb.paged_attention_forward(*args, cut.to(DEV), split=split)
    tsb.check_errors()
    assert torch.equal(out, expected)
    _check(out, oracle.paged_attention_decode(q, kc, vc, bt, 16, cut), "cut length")


def test_workspace_too_small_is_rejected():
    q, kc, vc, bt, sl = _paged_inputs([1300], 8, 2, 128, 16, torch.bfloat16, seed=5)
    ws = torch.empty(4, dtype=torch.float32, device=DEV)
    with pytest.raises(ValueError):
        tsb.paged_attention_forward(q.to(DEV), kc.to(DEV), vc.to(DEV), bt.to(DEV), 16,
                                    sl.to(DEV), workspace=ws)
    # (num_seqs * Hq * partitions * (head_dim + 2)) fp32 values; one sequence
    # splits into the shortest (256-key) partitions, a large batch into 2048-key ones
    assert tsb.paged_attention_workspace_bytes(1, 8, 128, 1300) == 1 * 8 * 6 * 130 * 4
    assert tsb.paged_attention_workspace_bytes(1, 8, 128, 256) == 0  # nothing to split
    assert tsb.paged_attention_workspace_bytes(512, 32, 128, 8192) == 512 * 32 * 4 * 130 * 4


def test_benchmark_step_against_fp32_attention():
    """The benchmark's own c3 decode step (256 sequences, 1.04 M context
    tokens, Qwen3-8B heads, 16-token pages in a 32768-block cache) against
    plain PyTorch attention in fp32 on the GPU over K/V gathered from each
    sequence's pages: the bf16 contract, >= 95% of elements bit-exact."""
    import torch.nn.functional as F

    from tinyserver_b200 import workloads as W

    cfg = W.CONFIGS["c3"]
    s = cfg.shape
    b = W.index_data(cfg, shard=0)
    lens = (b.positions + 1).to(torch.int32)
    S, Hq, Hkv, D, B = len(b.seqs), s.num_q_heads, s.num_kv_heads, s.head_dim, cfg.block_size
    g = torch.Generator(device=DEV).manual_seed(W.seed_of(cfg, 0) + 5)
    pool = torch.randn(2, cfg.num_blocks, Hkv, B, D, generator=g, device=DEV,
                       dtype=torch.float32).to(cfg.dtype)
    q = torch.randn(S, Hq, D, generator=g, device=DEV, dtype=torch.float32).to(cfg.dtype)
    bt = b.block_tables.to(DEV)
    out = tsb.paged_attention_forward(q, pool[0], pool[1], bt, B, lens.to(DEV))
    tsb.check_errors()
    expected = torch.empty_like(out)
    for i in range(S):
        L = int(lens[i])
        blocks = bt[i, :(L + B - 1) // B].long()
        kk = pool[0][blocks].permute(1, 0, 2, 3).reshape(Hkv, -1, D)[:, :L].float()
        vv = pool[1][blocks].permute(1, 0, 2, 3).reshape(Hkv, -1, D)[:, :L].float()
        kk = kk.repeat_interleave(Hq // Hkv, 0)[None]
        vv = vv.repeat_interleave(Hq // Hkv, 0)[None]
        o = F.scaled_dot_product_attention(q[i].float()[None, :, None, :], kk, vv)
        expected[i] = o[0, :, 0, :].to(cfg.dtype)
    _check(out, expected, "c3 decode step vs fp32 attention", min_exact=0.95)
