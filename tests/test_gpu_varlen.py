"""Prefill varlen attention on the GPU against the reference's own kernel
outputs (fp32 golden vectors) and the CPU oracle (16-bit types).

Tolerances: fp32 |a - e| <= 1e-4 + 1e-4 |e|; 16-bit outputs: the bf16/fp16
contract of tests/common.py.  Both 16-bit kernels round the probabilities to
the value dtype at the same point as the reference (before P V), but against
a different running max than the reference's 32-key blocks:
  * head_dim 64, the mma.sync kernel: 64-key tiles softmaxed in 32-key halves,
    >= 90% of elements bit-exact;
  * head_dim 128, the tcgen05 kernel: 128-key blocks, and a row's reference
    max moves only when the row max grows by more than 2^8 (so P may be scaled
    by up to 256 before rounding; O / l is unchanged).  Its rounding points
    are the reference's but its roundings differ, so instead of a bit-exact
    share it must be as accurate as the reference: against exact attention
    (fp32 math, P unrounded), its mean error at most 1.25x and its largest
    error at most 2x the reference algorithm's own (the oracle in 16 bits).
Every element of both is within the stated tolerance.
"""

import pytest
import torch

import tinyserver_b200 as tsb
from oracle import oracle
from tests.common import assert_close, load_golden

pytestmark = pytest.mark.gpu
DEV = "cuda"


def test_reference_golden_cases_fp32():
    g = load_golden("varlen_attention.pt")
    for c in g["cases"]:
        cu = c["cu_seqlens"].to(DEV)
        out = tsb.flash_attn_varlen_func(c["q"].to(DEV), c["k"].to(DEV), c["v"].to(DEV), cu, cu,
                                         c["max_seqlen"], c["max_seqlen"], c["causal"])
        torch.testing.assert_close(out.cpu(), c["out"], atol=1e-4, rtol=1e-4, msg=c["name"])


def _packed(lens, hq, hkv, hd, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    T = sum(lens)
    q = torch.randn(T, hq, hd, generator=g).to(dtype)
    k = torch.randn(T, hkv, hd, generator=g).to(dtype)
    v = torch.randn(T, hkv, hd, generator=g).to(dtype)
    cu = torch.zeros(len(lens) + 1, dtype=torch.int32)
    cu[1:] = torch.cumsum(torch.tensor(lens), 0)
    return q, k, v, cu


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("hq,hkv", [(4, 4), (8, 2), (16, 8), (32, 4)])
@pytest.mark.parametrize("hd", [64, 128])
@pytest.mark.parametrize("causal", [True, False])
def test_16bit_against_oracle(dtype, hq, hkv, hd, causal):
    lens = [1, 7, 63, 64, 65, 130, 333]
    q, k, v, cu = _packed(lens, hq, hkv, hd, dtype, seed=hq * 10 + hd + causal)
    expected = oracle.varlen_attention(q, k, v, cu, cu, causal)
    out = tsb.flash_attn_varlen_func(q.to(DEV), k.to(DEV), v.to(DEV), cu.to(DEV), cu.to(DEV),
                                     max(lens), max(lens), causal)
    assert out.shape == q.shape and out.dtype == q.dtype
    tsb.check_errors()
    assert_close(out, expected, f"{dtype} {hq}/{hkv} d{hd} causal={causal}",
                 min_exact=_min_exact(hd))
    if hd == 128:
        _as_accurate_as_reference(out, q, k, v, cu, cu, causal, f"{dtype} {hq}/{hkv} {causal}")


def _min_exact(hd):
    return 0.9 if hd == 64 else 0.0


def _as_accurate_as_reference(out, q, k, v, cq, ck, causal, what):
    """The tcgen05 path's error against exact attention is no worse than the
    reference algorithm's (see the module docstring)."""
    exact = oracle.varlen_attention(q.float(), k.float(), v.float(), cq, ck, causal)
    ref = oracle.varlen_attention(q, k, v, cq, ck, causal).float()
    e_out = (out.float().cpu() - exact).abs()
    e_ref = (ref - exact).abs()
    assert e_out.mean() <= 1.25 * e_ref.mean() + 1e-6, \
        f"{what}: mean error {float(e_out.mean()):.3e} vs reference {float(e_ref.mean()):.3e}"
    assert e_out.max() <= 2 * e_ref.max() + 1e-6, \
        f"{what}: max error {float(e_out.max()):.3e} vs reference {float(e_ref.max()):.3e}"


def test_views_of_a_merged_projection_at_qwen3_8b_heads():
    """q, k, v as strided head views of one (T, (Hq + 2 Hkv) * D) projection
    output, the layout the model produces (qwen3.py:264-266), one 192-token
    prefill chunk and a 1000-token sequence."""
    lens = [192, 1000]
    hq, hkv, hd = 32, 8, 128
    g = torch.Generator().manual_seed(3)
    T = sum(lens)
    qkv = torch.randn(T, (hq + 2 * hkv) * hd, generator=g).to(torch.bfloat16)
    q = qkv[:, :hq * hd].view(T, hq, hd)
    k = qkv[:, hq * hd:(hq + hkv) * hd].view(T, hkv, hd)
    v = qkv[:, (hq + hkv) * hd:].view(T, hkv, hd)
    cu = torch.tensor([0, 192, 1192], dtype=torch.int32)
    expected = oracle.varlen_attention(q.contiguous(), k.contiguous(), v.contiguous(), cu, cu,
                                       True)
    d = qkv.to(DEV)
    out = tsb.flash_attn_varlen_func(d[:, :hq * hd].view(T, hq, hd),
                                     d[:, hq * hd:(hq + hkv) * hd].view(T, hkv, hd),
                                     d[:, (hq + hkv) * hd:].view(T, hkv, hd), cu.to(DEV),
                                     cu.to(DEV), 1000, 1000, True)
    tsb.check_errors()
    assert_close(out, expected, "merged-projection views", min_exact=_min_exact(hd))
    _as_accurate_as_reference(out, q.contiguous(), k.contiguous(), v.contiguous(), cu, cu, True,
                              "merged-projection views")


@pytest.mark.parametrize("causal", [True, False])
def test_long_sequences_many_blocks_gqa(causal):
    """Qwen3-1.7B heads, sequences of several 256-query CTAs and many 128-key
    blocks, lengths that end inside a block and inside the second tile."""
    lens = [1024, 1500, 2047, 129]
    q, k, v, cu = _packed(lens, 16, 8, 128, torch.bfloat16, seed=40 + causal)
    expected = oracle.varlen_attention(q, k, v, cu, cu, causal)
    out = tsb.flash_attn_varlen_func(q.to(DEV), k.to(DEV), v.to(DEV), cu.to(DEV), cu.to(DEV),
                                     max(lens), max(lens), causal)
    tsb.check_errors()
    assert torch.isfinite(out).all()
    assert_close(out, expected, f"long causal={causal}", min_exact=0.0)
    _as_accurate_as_reference(out, q, k, v, cu, cu, causal, f"long causal={causal}")


def test_fewer_keys_than_queries():
    """Separate key lengths: the causal rule keeps key j for query i <= j's
    index within the sequence (top-left aligned), as the reference's mask."""
    g = torch.Generator().manual_seed(8)
    lq, lk = [300, 40], [100, 280]
    q = torch.randn(sum(lq), 8, 128, generator=g).to(torch.bfloat16)
    k = torch.randn(sum(lk), 4, 128, generator=g).to(torch.bfloat16)
    v = torch.randn(sum(lk), 4, 128, generator=g).to(torch.bfloat16)
    cq = torch.tensor([0, 300, 340], dtype=torch.int32)
    ck = torch.tensor([0, 100, 380], dtype=torch.int32)
    for causal in (False, True):
        expected = oracle.varlen_attention(q, k, v, cq, ck, causal)
        out = tsb.flash_attn_varlen_func(q.to(DEV), k.to(DEV), v.to(DEV), cq.to(DEV), ck.to(DEV),
                                         300, 280, causal)
        tsb.check_errors()
        assert_close(out, expected, f"lq != lk causal={causal}", min_exact=0.0)
        _as_accurate_as_reference(out, q, k, v, cq, ck, causal, f"lq != lk causal={causal}")


@pytest.mark.parametrize("scale", [0.25, -0.05, 0.0])
def test_softmax_scale_any_sign(scale):
    """An explicit softmax_scale, negative and zero included (the row max is
    taken after scaling, as the reference's), at head_dim 128."""
    lens = [5, 200, 300]
    q, k, v, cu = _packed(lens, 8, 4, 128, torch.bfloat16, seed=int(scale * 100) + 50)
    expected = oracle.varlen_attention(q, k, v, cu, cu, True, softmax_scale=scale)
    out = tsb.flash_attn_varlen_func(q.to(DEV), k.to(DEV), v.to(DEV), cu.to(DEV), cu.to(DEV),
                                     max(lens), max(lens), True, softmax_scale=scale)
    tsb.check_errors()
    assert torch.isfinite(out).all()
    assert_close(out, expected, f"scale={scale}", min_exact=0.0)


def _via_capi(q, k, v, cu, max_len, causal, counter):
    """One call through the C ABI with or without a work counter."""
    from tinyserver_b200 import _capi
    from tinyserver_b200._runtime import status_word, stream_ptr

    out = torch.empty_like(q)
    a = _capi.VarlenAttentionArgs()
    a.q, a.q_stride_token, a.q_stride_head = q.data_ptr(), q.stride(0), q.stride(1)
    a.k, a.k_stride_token, a.k_stride_head = k.data_ptr(), k.stride(0), k.stride(1)
    a.v, a.v_stride_token, a.v_stride_head = v.data_ptr(), v.stride(0), v.stride(1)
    a.out, a.out_stride_token, a.out_stride_head = out.data_ptr(), out.stride(0), out.stride(1)
    a.cu_seqlens_q = a.cu_seqlens_k = cu.data_ptr()
    a.batch, a.max_seqlen_q = cu.numel() - 1, max_len
    a.num_q_heads, a.num_kv_heads, a.head_dim = q.shape[1], k.shape[1], q.shape[2]
    a.causal = int(causal)
    a.scale = q.shape[2] ** -0.5
    a.dtype = _capi.QF_BF16
    a.status = status_word(q.device).data_ptr()
    a.total_q, a.total_k = q.shape[0], k.shape[0]
    a.work_counter = None if counter is None else counter.data_ptr()
    _capi.check(_capi.lib().qf_varlen_attention(a, stream_ptr(q.device)), "varlen")
    return out


@pytest.mark.parametrize("lens", [[3000, 40, 900, 1], [130] * 3, [2048] * 40])
def test_persistent_schedule_matches_one_cta_per_item(lens):
    """Persistent CTAs claiming items from a counter compute each item exactly
    as a CTA of its own would (bit-identical outputs), over fewer items than
    SMs, and many more; the counter is back at zero after every call, so the
    next call on the same counter sees all items again."""
    q, k, v, cu = _packed(lens, 16, 8, 128, torch.bfloat16, seed=len(lens))
    q, k, v, cu = q.to(DEV), k.to(DEV), v.to(DEV), cu.to(DEV)
    one = _via_capi(q, k, v, cu, max(lens), True, None)
    counter = torch.zeros(2, dtype=torch.int32, device=DEV)
    for _ in range(3):
        out = _via_capi(q, k, v, cu, max(lens), True, counter)
        tsb.check_errors()
        assert torch.equal(out, one)
        assert counter.tolist() == [0, 0]


@pytest.mark.parametrize("step", [128, 64, 32])
@pytest.mark.parametrize("scale", [1.0, 3.0])
def test_large_scores_growing_across_blocks(scale, step):
    """Scores whose row max grows by far more than 2^8 (and 2^32) from one
    run of `step` keys to the next: from block to block (128), from the first
    64 keys of a block to the last 64 (64), and from quarter to quarter (32).
    Covers the one-pass softmax's lazy rescale and its recompute path for
    rows whose probabilities would overflow, in either half of a block."""
    lens = [700, 300]
    q, k, v, cu = _packed(lens, 8, 4, 128, torch.bfloat16, seed=int(scale * 10) + 70 + step)
    # every run of `step` keys larger than the run before
    pos = torch.cat([torch.arange(n) for n in lens])
    k = (k.float() * (1.0 + (pos // step).float() * (step / 128)).view(-1, 1, 1)).to(torch.bfloat16)
    expected = oracle.varlen_attention(q, k, v, cu, cu, True, softmax_scale=scale)
    out = tsb.flash_attn_varlen_func(q.to(DEV), k.to(DEV), v.to(DEV), cu.to(DEV), cu.to(DEV),
                                     max(lens), max(lens), True, softmax_scale=scale)
    tsb.check_errors()
    assert torch.isfinite(out).all()
    assert_close(out, expected, f"growing scores scale={scale} step={step}", min_exact=0.0)


def test_cuda_graph_replays():
    """Captured once, replayed several times on new inputs: the persistent
    kernel's work counter is back at zero after every launch, so replays need
    no reset and match eager calls bit for bit."""
    lens = [700, 128, 1500, 3]
    q, k, v, cu = _packed(lens, 16, 8, 128, torch.bfloat16, seed=90)
    q, k, v, cu = q.to(DEV), k.to(DEV), v.to(DEV), cu.to(DEV)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        tsb.flash_attn_varlen_func(q, k, v, cu, cu, max(lens), max(lens), True)  # warm-up
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = tsb.flash_attn_varlen_func(q, k, v, cu, cu, max(lens), max(lens), True)
    for i in range(3):
        q.copy_(_packed(lens, 16, 8, 128, torch.bfloat16, seed=91 + i)[0].to(DEV))
        g.replay()
        torch.cuda.synchronize()
        eager = tsb.flash_attn_varlen_func(q, k, v, cu, cu, max(lens), max(lens), True)
        tsb.check_errors()
        assert torch.equal(out, eager), f"replay {i}"


def test_two_graphs_replay_only_the_second():
    """Two graphs captured one after the other (torch captures both on one
    shared capture stream); only the second is replayed.  A work counter made
    during a capture is zeroed only by that graph, so each capture must get a
    counter of its own rather than share one whose zero fill lives in the
    other graph."""
    lens = [513, 64, 1029]
    q, k, v, cu = _packed(lens, 16, 8, 128, torch.bfloat16, seed=95)
    q, k, v, cu = q.to(DEV), k.to(DEV), v.to(DEV), cu.to(DEV)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        tsb.flash_attn_varlen_func(q, k, v, cu, cu, max(lens), max(lens), True)  # warm-up
    torch.cuda.current_stream().wait_stream(s)
    graphs, outs = [], []
    for _ in range(2):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            outs.append(tsb.flash_attn_varlen_func(q, k, v, cu, cu, max(lens), max(lens), True))
        graphs.append(g)
    eager = tsb.flash_attn_varlen_func(q, k, v, cu, cu, max(lens), max(lens), True)
    for i in range(3):
        graphs[1].replay()
        torch.cuda.synchronize()
        tsb.check_errors()
        assert torch.equal(outs[1], eager), f"second graph, replay {i}"
    del graphs


@pytest.mark.parametrize("causal", [True, False])
def test_empty_sequences_keyless_rows_and_many_short(causal):
    """Edge cases of the packed layout on the tensor-core path: zero-length
    sequences between others, a sequence whose queries have no keys (0 / 0,
    NaN rows, as the reference's acc / l), and 600 short sequences (many more
    work items than SMs, most with one tile)."""
    g = torch.Generator().manual_seed(120 + causal)
    lq = [3, 0, 130, 0, 1, 9, 300]
    lk = [3, 0, 130, 0, 1, 0, 300]  # the sixth sequence: 9 queries, no keys
    q = torch.randn(sum(lq), 8, 128, generator=g).to(torch.bfloat16)
    k = torch.randn(sum(lk), 2, 128, generator=g).to(torch.bfloat16)
    v = torch.randn(sum(lk), 2, 128, generator=g).to(torch.bfloat16)
    cq = torch.tensor([0] + torch.tensor(lq).cumsum(0).tolist(), dtype=torch.int32)
    ck = torch.tensor([0] + torch.tensor(lk).cumsum(0).tolist(), dtype=torch.int32)
    expected = oracle.varlen_attention(q, k, v, cq, ck, causal)
    out = tsb.flash_attn_varlen_func(q.to(DEV), k.to(DEV), v.to(DEV), cq.to(DEV), ck.to(DEV),
                                     max(lq), max(lk), causal).cpu()
    tsb.check_errors()
    nan_e, nan_o = torch.isnan(expected.float()), torch.isnan(out.float())
    assert nan_e.any() and torch.equal(nan_e, nan_o)
    keep = ~nan_e.flatten(1).any(1)
    assert_close(out[keep], expected[keep], f"empty / keyless causal={causal}", min_exact=0.0)

    lens = torch.randint(1, 41, (600,), generator=g).tolist()
    q, k, v, cu = _packed(lens, 8, 2, 128, torch.bfloat16, seed=130 + causal)
    expected = oracle.varlen_attention(q, k, v, cu, cu, causal)
    out = tsb.flash_attn_varlen_func(q.to(DEV), k.to(DEV), v.to(DEV), cu.to(DEV), cu.to(DEV),
                                     max(lens), max(lens), causal)
    tsb.check_errors()
    assert_close(out, expected, f"600 short causal={causal}", min_exact=0.0)
    _as_accurate_as_reference(out, q, k, v, cu, cu, causal, f"600 short causal={causal}")


def test_benchmark_batch_against_fp32_attention():
    """The benchmark's own c2 batch (16 sequences, 14,611 tokens, Qwen3-1.7B
    heads) through the tensor-core path, checked sequence by sequence against
    plain PyTorch attention in fp32 on the GPU (GQA heads expanded, causal):
    every element within the bf16 contract, and the mean error small."""
    import torch.nn.functional as F

    from tinyserver_b200 import workloads as W

    cfg = W.CONFIGS["c2"]
    s = cfg.shape
    lens = [n for n, _ in W.sequences(cfg, 0)]
    T, Hq, Hkv, D = sum(lens), s.num_q_heads, s.num_kv_heads, s.head_dim
    g = torch.Generator(device=DEV).manual_seed(W.seed_of(cfg, 0) + 9)
    q = torch.randn(T, Hq, D, generator=g, device=DEV).to(cfg.dtype)
    k = torch.randn(T, Hkv, D, generator=g, device=DEV).to(cfg.dtype)
    v = torch.randn(T, Hkv, D, generator=g, device=DEV).to(cfg.dtype)
    cu = torch.zeros(len(lens) + 1, dtype=torch.int32)
    cu[1:] = torch.cumsum(torch.tensor(lens), 0)
    out = tsb.flash_attn_varlen_func(q, k, v, cu.to(DEV), cu.to(DEV), max(lens), max(lens),
                                     True)
    tsb.check_errors()
    expected = torch.empty_like(out)
    for b in range(len(lens)):
        a0, a1 = int(cu[b]), int(cu[b + 1])
        qs = q[a0:a1].float().transpose(0, 1)[None]
        ks = k[a0:a1].float().transpose(0, 1).repeat_interleave(Hq // Hkv, 0)[None]
        vs = v[a0:a1].float().transpose(0, 1).repeat_interleave(Hq // Hkv, 0)[None]
        o = F.scaled_dot_product_attention(qs, ks, vs, is_causal=True)
        expected[a0:a1] = o[0].transpose(0, 1).to(cfg.dtype)
    assert_close(out, expected, "c2 batch vs fp32 attention", min_exact=0.0)
    err = (out.float() - expected.float()).abs().mean().item()
    assert err < 2e-3, f"mean abs error {err:.3e}"


def test_concurrent_streams_use_separate_work_counters():
    """Calls on two streams may run at the same time on the GPU; each stream
    gets its own work counter, so both results match single-stream calls bit
    for bit."""
    lens = [900, 1500, 300]
    ins = []
    for seed in (150, 151):
        q, k, v, cu = _packed(lens, 16, 8, 128, torch.bfloat16, seed=seed)
        ins.append((q.to(DEV), k.to(DEV), v.to(DEV), cu.to(DEV)))
    ref = [tsb.flash_attn_varlen_func(q, k, v, cu, cu, max(lens), max(lens), True)
           for q, k, v, cu in ins]
    torch.cuda.synchronize()
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    outs = [None, None]
    for rep in range(3):
        for i, st in enumerate(streams):
            st.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(st):
                q, k, v, cu = ins[i]
                outs[i] = tsb.flash_attn_varlen_func(q, k, v, cu, cu, max(lens), max(lens), True)
        torch.cuda.synchronize()
        tsb.check_errors()
        for i in range(2):
            assert torch.equal(outs[i], ref[i]), f"stream {i}, repetition {rep}"
