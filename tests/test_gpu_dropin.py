"""The drop-in boundary end to end on the GPU: a seeded random-init
transformers Qwen3 model with the fused ops installed, against the same model
unpatched.

* Module level (``install_fused(paged=False)`` + ``apply_rotary_pos_emb``
  override): the stock HF attention path with fused embedding, norms,
  add+norm and SiLU-and-mul.
* Paged: the reference's batch format (flattened prefill of two sequences,
  then a decode step), the fused q_norm/k_norm + RoPE + KV-store launch per
  layer and an attention backend that reads K and V back OUT OF THE PAGED
  CACHE -- so the logits only match if every row landed in its slot.  The
  expected logits come from the unpatched model run on each sequence alone.

Tolerance: logits of a 2-layer bf16 model; the fused RMS reductions sum in a
different order than torch, which moves a bf16 rounding now and then, so the
check is |a - e| <= 0.05 + 0.02 |e| on the logits plus an identical argmax.
"""

import pytest
import torch

import tinyserver_b200 as tsb
from tests.qwen3_tiny import Context, block_tables, clone, tiny_model
from tinyserver_b200 import patches

pytestmark = pytest.mark.gpu
DEV = "cuda"
ATOL, RTOL = 0.05, 0.02


def _close(a, e, what):
    a, e = a.float().cpu(), e.float().cpu()
    err = (a - e).abs()
    assert (err <= ATOL + RTOL * e.abs()).all(), f"{what}: max err {float(err.max()):.4f}"
    assert torch.equal(a.argmax(-1), e.argmax(-1)), f"{what}: argmax differs"


def _stock_logits(model, ids):
    with torch.no_grad():
        T = ids.shape[-1]
        return model(input_ids=ids.view(1, T), position_ids=torch.arange(T, device=DEV)[None],
                     use_cache=False).logits[0]


class CacheSdpa:
    """Test attention backend: SDPA over K/V gathered from the paged cache."""

    def prefill(self, q, k, v, m, attn):
        outs = []
        cu = m.cu_seqlens.tolist()
        for s in range(len(cu) - 1):
            t0, t1 = cu[s], cu[s + 1]
            bm, sm = m.block_mapping[t0:t1], m.slot_mapping[t0:t1]
            kc = attn.k_cache[bm, :, sm, :]  # (n, Hkv, D) read back from the pages
            vc = attn.v_cache[bm, :, sm, :]
            assert torch.equal(kc, k[t0:t1]) and torch.equal(vc, v[t0:t1])
            o = torch.nn.functional.scaled_dot_product_attention(
                q[t0:t1].transpose(0, 1)[None], kc.transpose(0, 1)[None],
                vc.transpose(0, 1)[None], is_causal=True, enable_gqa=True,
                scale=q.shape[-1] ** -0.5)
            outs.append(o[0].transpose(0, 1).reshape(t1 - t0, -1))
        return torch.cat(outs)

    def decode(self, q, m, attn):
        B = attn.k_cache.shape[2]
        outs = []
        for s in range(q.shape[0]):
            L = int(m.seq_lens[s])
            pos = torch.arange(L, device=q.device)
            blocks = m.block_tables[s].long()[pos // B]
            kc = attn.k_cache[blocks, :, pos % B, :]
            vc = attn.v_cache[blocks, :, pos % B, :]
            o = torch.nn.functional.scaled_dot_product_attention(
                q[s:s + 1].transpose(0, 1)[None], kc.transpose(0, 1)[None],
                vc.transpose(0, 1)[None], enable_gqa=True, scale=q.shape[-1] ** -0.5)
            outs.append(o[0].transpose(0, 1).reshape(1, -1))
        return torch.cat(outs)


@pytest.fixture(scope="module")
def stock():
    return tiny_model(device=DEV)


def test_module_level_install_matches_stock(stock):
    fused = patches.install_fused(clone(stock), paged=False)
    ids = torch.randint(0, 512, (96,), generator=torch.Generator().manual_seed(1)).to(DEV)
    expected = _stock_logits(stock, ids)
    try:
        patches.install_operator_overrides()
        got = _stock_logits(fused, ids)
    finally:
        patches.restore_operator_overrides()
    tsb.check_errors()
    _close(got, expected, "module-level install")


@pytest.mark.parametrize("decode", ["sdpa-from-cache", "fused-kernel", "fused-prefill-and-decode"])
@pytest.mark.parametrize("block_size", [16, 4])
def test_paged_prefill_then_decode_matches_stock(stock, block_size, decode):
    lens = [37, 64]
    num_blocks = 128
    blocks_each = (max(lens) + 1 + block_size - 1) // block_size
    tables = block_tables(len(lens), blocks_each, num_blocks)
    fused = clone(stock)
    pool = patches.allocate_kv_cache(fused, num_blocks, block_size, torch.bfloat16, DEV)
    pool.normal_()  # poisoned: rows the batch does not write must stay as they are
    poisoned = pool.clone()
    ctx = Context()
    backend = {"sdpa-from-cache": CacheSdpa(),
               "fused-kernel": patches.FusedDecodeAttention(prefill=CacheSdpa()),
               "fused-prefill-and-decode": patches.FusedDecodeAttention()}[decode]
    patches.install_fused(fused, context=lambda: ctx, attention=backend)

    g = torch.Generator().manual_seed(5)
    seqs = [torch.randint(0, 512, (n,), generator=g).to(DEV) for n in lens]
    # prefill: flattened batch, positions restart per sequence
    ids = torch.cat(seqs)[None]
    pos = torch.cat([torch.arange(n, device=DEV) for n in lens])[None]
    ctx.mode = "prefill"
    ctx.sequences = [{"num_tokens": n, "block_table": t} for n, t in zip(lens, tables)]
    with torch.no_grad():
        logits = fused(input_ids=ids, position_ids=pos, use_cache=False).logits[0]
    tsb.check_errors()
    t0 = 0
    for s, n in enumerate(lens):
        _close(logits[t0:t0 + n], _stock_logits(stock, seqs[s]), f"prefill seq {s}")
        t0 += n

    # untouched slots: everything outside the written (block, slot) pairs
    written = torch.zeros(num_blocks, block_size, dtype=torch.bool)
    for n, t in zip(lens, tables):
        for p in range(n):
            written[t[p // block_size], p % block_size] = True
    keep = ~written.to(DEV)
    assert torch.equal(pool.transpose(3, 4)[:, :, keep], poisoned.transpose(3, 4)[:, :, keep])

    # decode: one new token per sequence at position len
    nxt = torch.stack([logits[sum(lens[:s + 1]) - 1].argmax() for s in range(len(lens))])
    ctx.mode = "decode"
    with torch.no_grad():
        dec = fused(input_ids=nxt[None], position_ids=torch.tensor([lens], device=DEV),
                    use_cache=False).logits[0]
    tsb.check_errors()
    for s, n in enumerate(lens):
        full = torch.cat([seqs[s], nxt[s:s + 1]])
        _close(dec[s], _stock_logits(stock, full)[-1], f"decode seq {s}")
