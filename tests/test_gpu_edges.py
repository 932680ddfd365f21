"""Edge cases of the CUDA path: empty and ragged batches, odd layouts and
dtypes, strided caches, int32/int64 indices, and out-of-range indices (which
the kernels must skip and report, never write)."""

import pytest
import torch

import tinyserver_b200 as tsb
from oracle import oracle
from tests.common import assert_close

pytestmark = pytest.mark.gpu
DEV = "cuda"


def rnd(*shape, dtype=torch.bfloat16, seed=0):
    g = torch.Generator(device=DEV).manual_seed(seed)
    return torch.randn(*shape, generator=g, device=DEV).to(dtype)


@pytest.fixture(autouse=True)
def _clean_flags():
    tsb.check_errors()
    yield


def test_empty_batches_launch_nothing():
    H, D = 256, 128
    x = rnd(0, H)
    w = rnd(H)
    assert tsb.rms_norm(x, w, 1e-6).shape == (0, H)
    y, h = tsb.fused_add_rms_norm(x, x, w, 1e-6)
    assert y.shape == (0, H)
    assert tsb.silu_and_mul(rnd(0, 2 * H)).shape == (0, H)
    assert tsb.embedding(torch.zeros(0, dtype=torch.long, device=DEV), rnd(10, H)).shape == (0, H)
    kc = rnd(4, 2, 16, D)
    before = kc.clone()
    tsb.store_kv_cache_batched(rnd(2, 0, D), rnd(2, 0, D), kc, kc.clone(),
                               torch.zeros(0, dtype=torch.long, device=DEV),
                               torch.zeros(0, dtype=torch.long, device=DEV))
    assert torch.equal(kc, before)
    q = rnd(0, 4, D)
    qo, ko = tsb.qk_norm_rope_store(q, rnd(0, 2, D), None, rnd(D), rnd(D), 1e-6, rnd(0, D),
                                    rnd(0, D))
    assert qo.shape == (0, 4, D)
    tsb.check_errors()


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("H", [8, 200, 1000, 1024, 4096, 5120, 8192])
@pytest.mark.parametrize("T", [1, 3, 1000])
def test_rmsnorm_shapes(dtype, H, T):
    x, r, w = rnd(T, H, dtype=dtype, seed=1), rnd(T, H, dtype=dtype, seed=2), rnd(H, dtype=dtype)
    y, h = tsb.fused_add_rms_norm(x, r, w, 1e-6)
    ry, rh = oracle.add_rmsnorm(x.cpu(), r.cpu(), w.cpu(), 1e-6)
    assert torch.equal(h.cpu(), rh)
    assert_close(y, ry, f"add_rmsnorm {dtype} H={H}", min_exact=0.98)
    assert_close(tsb.rms_norm(x, w, 1e-6), oracle.rmsnorm(x.cpu(), w.cpu(), 1e-6), "rmsnorm",
                 min_exact=0.98)


def test_rmsnorm_odd_hidden_and_strided_rows():
    """Hidden sizes that are not a multiple of 8 and rows with padding take
    the scalar kernel."""
    for H in (7, 33, 1001):
        base = rnd(5, H + 3, seed=H)
        x = base[:, :H]  # row stride H+3: not 16-byte aligned rows
        w = rnd(H, seed=1)
        assert_close(tsb.rms_norm(x, w, 1e-5), oracle.rmsnorm(x.cpu(), w.cpu(), 1e-5),
                     f"rmsnorm H={H}", min_exact=0.98)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("I", [4, 12, 100, 3072, 25600])
def test_silu_shapes(dtype, I):
    gu = rnd(17, 2 * I, dtype=dtype, seed=I) * 4
    out = tsb.silu_and_mul(gu)
    ref = oracle.silu_and_mul(gu[:, :I].cpu(), gu[:, I:].cpu())
    assert_close(out, ref, f"silu {dtype} I={I}", min_exact=0.98)


def test_silu_extreme_values():
    g = torch.tensor([[-1e4, -100., -88., -20., -1., -0., 0., 1e-30, 1., 20., 88., 100.,
                       1e4, 3e38, -3e38, 0.5]], device=DEV)
    u = torch.ones_like(g)
    for dt in (torch.float32, torch.bfloat16):
        out = tsb.silu_and_mul(g.to(dt), u.to(dt))
        ref = oracle.silu_and_mul(g.to(dt).cpu(), u.to(dt).cpu())
        assert torch.isfinite(out).all()
        assert_close(out, ref, f"silu extremes {dt}")


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_embedding_int32_int64_and_odd_rows(dtype):
    table = rnd(1000, 96, dtype=dtype)
    ids = torch.tensor([0, 999, 5, 5, 123], device=DEV)
    for it in (torch.int32, torch.int64):
        assert torch.equal(tsb.embedding(ids.to(it), table), table[ids])
    odd = rnd(50, 7, dtype=dtype)  # 14- or 28-byte rows: scalar path
    assert torch.equal(tsb.embedding(ids % 50, odd), odd[ids % 50])
    ids2 = ids.view(1, 5)
    assert tsb.embedding(ids2, table).shape == (1, 5, 96)


def test_embedding_out_of_range_is_flagged_not_read():
    table = rnd(100, 64)
    ids = torch.tensor([1, 100, -1, 2], device=DEV)
    out = tsb.embedding(ids, table)
    assert torch.equal(out[0], table[1]) and torch.equal(out[3], table[2])
    assert not out[1].any() and not out[2].any()
    with pytest.raises(IndexError, match="vocabulary"):
        tsb.check_errors()


@pytest.mark.parametrize("head_dim", [8, 16, 32, 128])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_store_reference_geometries(head_dim, dtype):
    """The head sizes of the reference's own store tests (8/16/32) plus 128,
    scattered into a poisoned cache."""
    Hkv, B, N, T = 4, 4, 9, 13
    k = rnd(Hkv, T, head_dim, dtype=dtype, seed=1)
    v = rnd(Hkv, T, head_dim, dtype=dtype, seed=2)
    slots = torch.randperm(N * B, generator=torch.Generator().manual_seed(3))[:T]
    bm, sm = (slots // B).to(DEV), (slots % B).to(DEV)
    kc, vc = rnd(N, Hkv, B, head_dim, dtype=dtype, seed=4), rnd(N, Hkv, B, head_dim,
                                                                  dtype=dtype, seed=5)
    rk, rv = kc.cpu(), vc.cpu()
    oracle.kv_store_batched(k.cpu(), v.cpu(), rk, rv, bm.cpu(), sm.cpu())
    tsb.store_kv_cache_batched(k, v, kc, vc, bm.to(torch.int32), sm.to(torch.int32))
    assert torch.equal(kc.cpu(), rk) and torch.equal(vc.cpu(), rv)


def test_store_non_contiguous_head_dim_takes_scalar_path():
    Hkv, T, D, N, B = 2, 5, 16, 4, 4
    base = rnd(Hkv, T, D, 2, seed=9)
    k = base[..., 0]  # head_dim stride 2
    v = base[..., 1]
    bm = torch.tensor([3, 3, 0, 1, 2], device=DEV)
    sm = torch.tensor([0, 1, 3, 2, 0], device=DEV)
    kc, vc = rnd(N, Hkv, B, D, seed=1), rnd(N, Hkv, B, D, seed=2)
    rk, rv = kc.cpu(), vc.cpu()
    oracle.kv_store_batched(k.cpu(), v.cpu(), rk, rv, bm.cpu(), sm.cpu())
    tsb.store_kv_cache_batched(k, v, kc, vc, bm, sm)
    assert torch.equal(kc.cpu(), rk) and torch.equal(vc.cpu(), rv)


def test_store_into_strided_layer_views_of_a_pool():
    """(2, L, N, Hkv, B, D) pool, layer 1 of 3: per-layer views are strided in
    the leading dims exactly as qwen3_cache_allocator makes them."""
    L, N, Hkv, B, D, T = 3, 6, 8, 16, 128, 40
    pool = rnd(2, L, N, Hkv, B, D, seed=11)
    before = pool.clone()
    k, v = rnd(Hkv, T, D, seed=12), rnd(Hkv, T, D, seed=13)
    slots = torch.randperm(N * B, generator=torch.Generator().manual_seed(1))[:T].to(DEV)
    tsb.store_kv_cache_batched(k, v, pool[0, 1], pool[1, 1], slots // B, slots % B)
    exp = before.clone()
    exp[0, 1, slots // B, :, slots % B] = k.transpose(0, 1)
    exp[1, 1, slots // B, :, slots % B] = v.transpose(0, 1)
    assert torch.equal(pool, exp)


def test_store_out_of_range_indices_are_skipped_and_flagged():
    Hkv, T, D, N, B = 2, 4, 128, 3, 16
    k, v = rnd(Hkv, T, D, seed=1), rnd(Hkv, T, D, seed=2)
    kc, vc = rnd(N, Hkv, B, D, seed=3), rnd(N, Hkv, B, D, seed=4)
    before_k, before_v = kc.clone(), vc.clone()
    bm = torch.tensor([0, 3, -1, 2], device=DEV)   # block 3 and -1 are outside
    sm = torch.tensor([1, 0, 0, 16], device=DEV)   # slot 16 is outside
    tsb.store_kv_cache_batched(k, v, kc, vc, bm, sm)
    with pytest.raises(IndexError):
        tsb.check_errors()
    exp_k = before_k.clone()
    exp_k[0, :, 1] = k[:, 0]
    assert torch.equal(kc, exp_k)
    exp_v = before_v.clone()
    exp_v[0, :, 1] = v[:, 0]
    assert torch.equal(vc, exp_v)
    # per-sequence entry: a position past the block table is skipped too
    tsb.store_kv_cache(16, torch.tensor([0], dtype=torch.int32, device=DEV), k[:, :1], v[:, :1],
                       kc, vc)
    with pytest.raises(IndexError, match="block table"):
        tsb.check_errors()
    assert torch.equal(kc, exp_k)


@pytest.mark.parametrize("head_dim", [64, 128, 256])
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_qk_norm_rope_head_dims(head_dim, dtype):
    T, Hq, Hkv = 37, 6, 2
    q, k, v = (rnd(T, Hq, head_dim, dtype=dtype, seed=1), rnd(T, Hkv, head_dim, dtype=dtype,
                                                               seed=2),
               rnd(T, Hkv, head_dim, dtype=dtype, seed=3))
    qw, kw = (1 + 0.02 * rnd(head_dim, seed=4).float()).to(dtype), \
        (1 + 0.02 * rnd(head_dim, seed=5).float()).to(dtype)
    pos = torch.randint(0, 40000, (T,), device=DEV)
    inv = tsb.rope_inv_freq(head_dim, 1e6, DEV)
    cos, sin = tsb.rope_cos_sin(pos, inv, head_dim, dtype)
    N, B = 10, 16
    kc, vc = rnd(N, Hkv, B, head_dim, dtype=dtype, seed=6), rnd(N, Hkv, B, head_dim,
                                                                  dtype=dtype, seed=7)
    slots = torch.randperm(N * B, generator=torch.Generator().manual_seed(8))[:T].to(DEV)
    qo, ko = tsb.qk_norm_rope_store(q, k, v, qw, kw, 1e-6, cos, sin, kc, vc, slots // B,
                                    slots % B)
    rq, rk = oracle.qk_norm_rope_store(q.cpu(), k.cpu(), None, qw.cpu(), kw.cpu(), 1e-6,
                                       cos.cpu(), sin.cpu())
    assert_close(qo, rq, "q", min_exact=0.98)
    assert_close(ko, rk, "k", min_exact=0.98)
    assert torch.equal(kc[slots // B, :, slots % B], ko)
    assert torch.equal(vc[slots // B, :, slots % B], v)
    # cos/sin computed in-kernel give the same bits as the table
    qo2, ko2 = tsb.qk_norm_rope_store(q, k, None, qw, kw, 1e-6, None, None, positions=pos,
                                      inv_freq=inv)
    assert torch.equal(qo2, qo) and torch.equal(ko2, ko)


def test_qk_store_bad_slot_is_flagged():
    T, Hq, Hkv, D = 3, 2, 2, 128
    q, k, v = rnd(T, Hq, D, seed=1), rnd(T, Hkv, D, seed=2), rnd(T, Hkv, D, seed=3)
    kc, vc = rnd(2, Hkv, 16, D, seed=4), rnd(2, Hkv, 16, D, seed=5)
    bk, bv = kc.clone(), vc.clone()
    cos, sin = tsb.rope_cos_sin(torch.arange(T, device=DEV), tsb.rope_inv_freq(D, 1e6, DEV), D,
                                torch.bfloat16)
    qo, ko = tsb.qk_norm_rope_store(q, k, v, None, None, 1e-6, cos, sin, kc, vc,
                                    torch.tensor([0, 2, 1], device=DEV),
                                    torch.tensor([5, 0, 99], device=DEV))
    with pytest.raises(IndexError):
        tsb.check_errors()
    bk[0, :, 5] = ko[0]
    bv[0, :, 5] = v[0]
    assert torch.equal(kc, bk) and torch.equal(vc, bv)


def test_build_slot_mapping_flags_positions_past_the_table():
    cu = torch.tensor([0, 2, 3], dtype=torch.int32, device=DEV)
    pos = torch.tensor([0, 17, 40], device=DEV)
    bt = torch.tensor([[5, 6], [7, 8]], dtype=torch.int32, device=DEV)
    bm, sm = tsb.build_slot_mapping(cu, pos, bt, 16)
    assert bm.tolist() == [5, 6, -1] and sm.tolist() == [0, 1, 0]
    with pytest.raises(IndexError, match="block table"):
        tsb.check_errors()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs on one box")
def test_ops_on_a_device_that_is_not_current():
    """Tensors on cuda:1 while cuda:0 is current: every op launches on the
    tensors' device (and the default stream of that device), not the current
    one, and leaves the current device as it was."""
    torch.cuda.set_device(0)
    d1 = torch.device("cuda", 1)
    g = torch.Generator(device=d1).manual_seed(5)
    x = torch.randn(64, 256, generator=g, device=d1).to(torch.bfloat16)
    w = torch.randn(256, generator=g, device=d1).to(torch.bfloat16)
    y = tsb.rms_norm(x, w, 1e-6)
    gu = torch.randn(64, 512, generator=g, device=d1).to(torch.bfloat16)
    act = tsb.silu_and_mul(gu)
    tsb.check_errors(d1)
    assert torch.cuda.current_device() == 0
    assert_close(y, oracle.rmsnorm(x.cpu(), w.cpu(), 1e-6), "rms_norm on cuda:1")
    assert_close(act, oracle.silu_and_mul(gu[:, :256].cpu(), gu[:, 256:].cpu()), "silu on cuda:1")
    lens = torch.tensor([37, 190], dtype=torch.int32)  # within the 12-block table rows
    q = torch.randn(2, 8, 128, generator=g, device=d1).to(torch.bfloat16)
    kc = torch.randn(24, 2, 16, 128, generator=g, device=d1).to(torch.bfloat16)
    vc = torch.randn(24, 2, 16, 128, generator=g, device=d1).to(torch.bfloat16)
    bt = torch.arange(24, dtype=torch.int32, device=d1).view(2, 12)
    out = tsb.paged_attention_forward(q, kc, vc, bt, 16, lens.to(d1))
    tsb.check_errors(d1)
    assert_close(out, oracle.paged_attention_decode(q.cpu(), kc.cpu(), vc.cpu(), bt.cpu(), 16,
                                                    lens), "decode on cuda:1", min_exact=0.98)
    assert torch.cuda.current_device() == 0
