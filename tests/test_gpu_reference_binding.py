"""The reference-side binding on the GPU: the reference's own loader, patched
attention forward, inference context and prefill helper, run unmodified from
its offline install (baseline/_ref, or TINYSERVER_REF; skipped without it),
with this library bound in the two ways a maintainer would bind it:

* ``fused_qwen3_model_loader`` in place of ``qwen3_model_loader``
  (server/model/hf_backend.py:16-18): the reference's cache allocator, then
  every fused op, attention on this library's kernels;
* the reference's ``qwen3_model_loader`` plus ``install_operator_overrides``:
  the reference's ``_page_attention_forward`` (server/model/patches/
  qwen3.py:216-418) calling this library's ``apply_rotary_pos_emb``,
  ``store_kv_cache_batched`` (prefill, :311) and ``store_kv_cache`` (decode,
  :350) by name.

Both run a prefill of three packed sequences built by the reference's
``build_prefill_inputs`` under its ``inference_context``, then a decode step
with the engine's decode context (engine.py:579-582), and are compared with the
unmodified reference model (its Triton store and attention kernels) on the
same weights: logits within |a - e| <= 0.05 + 0.02 |e| (the bf16 tolerance of
the drop-in tests) with the same argmax up to near-ties (at most 2% of the
rows, each pick's expected logit within that tolerance of the best); K pages
within the bf16 contract with >= 98% of elements bit-exact, V pages bit-exact
when the reference's own norms and projections feed them (operator
overrides); with the fused loader, layer 0's pages within the bf16 contract
(>= 98% bit-exact) and deeper layers' -- which see the earlier layers'
rounding differences -- within the logits' tolerance; and every slot the
batch did not write still zero, as the reference's allocator left it.
"""

import pytest
import torch

import tinyserver_b200 as tsb
from tests.common import assert_close, reference_module
from tests.qwen3_tiny import block_tables, clone, tiny_model
from tinyserver_b200 import patches

pytestmark = pytest.mark.gpu
DEV = "cuda"
ATOL, RTOL = 0.05, 0.02
BLOCK = 16


def _close(a, e, what):
    """Logits within tolerance, and the same argmax except on near-ties: where
    the picks differ, the expected logits of the two picks lie within the
    tolerance of each other (the reference's Triton attention and this
    library's round differently, which may swap two tokens that tie)."""
    a, e = a.float().cpu(), e.float().cpu()
    err = (a - e).abs()
    assert (err <= ATOL + RTOL * e.abs()).all(), f"{what}: max err {float(err.max()):.4f}"
    ia, ie = a.argmax(-1), e.argmax(-1)
    rows = (ia != ie).nonzero().flatten()
    best = e[rows, ie[rows]]
    gap = best - e[rows, ia[rows]]
    assert (gap <= ATOL + RTOL * best.abs()).all(), f"{what}: argmax differs beyond a near-tie"
    assert rows.numel() <= max(1, a.shape[0] // 50), f"{what}: {rows.numel()} argmax ties"


@pytest.fixture(scope="module")
def ref():
    return {name: reference_module(f"server.model.{name}")
            for name in ("patches.qwen3", "inference_context", "prefill_helpers")}


def _run(model, ref, seqs, tables, nxt=None):
    """Prefill (and, with ``nxt``, one decode step) through the reference's
    batch format; returns (prefill logits, decode logits or None)."""
    ctx_mod, helpers = ref["inference_context"], ref["prefill_helpers"]
    ids, pos, ctx = helpers.build_prefill_inputs([s.tolist() for s in seqs], tables, DEV)
    with torch.no_grad(), ctx_mod.inference_context(ctx):
        pre = model(input_ids=ids, position_ids=pos, use_cache=False).logits[0]
    dec = None
    if nxt is not None:
        dctx = ctx_mod.InferenceContext(mode="decode",
                                        sequences=[{"block_table": t} for t in tables])
        dpos = torch.tensor([[len(s) for s in seqs]], device=DEV)
        with torch.no_grad(), ctx_mod.inference_context(dctx):
            dec = model(input_ids=nxt[None], position_ids=dpos, use_cache=False).logits[0]
    return pre, dec


def _written(seqs, tables):
    bm, sm = [], []
    for s, t in zip(seqs, tables):
        for p in range(len(s) + 1):  # prefill rows and the decode row
            bm.append(t[p // BLOCK])
            sm.append(p % BLOCK)
    return torch.tensor(bm, device=DEV), torch.tensor(sm, device=DEV)


@pytest.mark.parametrize("binding", ["fused_loader", "operator_overrides"])
def test_reference_forward_with_the_library_bound(ref, binding):
    qwen3 = ref["patches.qwen3"]
    stock = tiny_model(device=DEV)
    expected_model, model = clone(stock), clone(stock)
    util = 0.002  # a few hundred MB of the GPU's free memory for each pool
    # the reference's allocator keeps room for the peak allocation seen so far
    # (server/model/utils.py get_available_memory); earlier tests' peaks are
    # not this model's
    torch.cuda.empty_cache()
    torch.cuda.reset_peak_memory_stats()
    n_ref = qwen3.qwen3_model_loader(expected_model, expected_model.config, util, BLOCK,
                                     torch.bfloat16, DEV)
    if binding == "fused_loader":
        n = patches.fused_qwen3_model_loader(model, model.config, util, BLOCK, torch.bfloat16,
                                             DEV)
    else:
        n = qwen3.qwen3_model_loader(model, model.config, util, BLOCK, torch.bfloat16, DEV)
    lens = [37, 64, 129]
    tables = block_tables(len(lens), (max(lens) + BLOCK) // BLOCK, min(n, n_ref, 512), seed=11)
    g = torch.Generator().manual_seed(21)
    seqs = [torch.randint(0, 512, (k,), generator=g).to(DEV) for k in lens]

    exp_pre, _ = _run(expected_model, ref, seqs, tables)
    nxt = torch.stack([exp_pre[sum(lens[:i + 1]) - 1].argmax() for i in range(len(lens))])
    exp_pre, exp_dec = _run(expected_model, ref, seqs, tables, nxt)
    if binding == "operator_overrides":
        try:
            patches.install_operator_overrides()
            pre, dec = _run(model, ref, seqs, tables, nxt)
        finally:
            patches.restore_operator_overrides()
    else:
        pre, dec = _run(model, ref, seqs, tables, nxt)
    tsb.check_errors()
    _close(pre, exp_pre, f"{binding}: prefill logits")
    _close(dec, exp_dec, f"{binding}: decode logits")

    bm, sm = _written(seqs, tables)
    for i, (layer, exp_layer) in enumerate(zip(model.model.layers, expected_model.model.layers)):
        a, e = layer.self_attn, exp_layer.self_attn
        ka, ke = a.k_cache[bm, :, sm, :], e.k_cache[bm, :, sm, :]
        va, ve = a.v_cache[bm, :, sm, :], e.v_cache[bm, :, sm, :]
        if binding == "operator_overrides":  # the reference's own norms and projections
            assert torch.equal(va, ve), f"layer {i}: V pages"
            assert_close(ka, ke, f"layer {i}: K pages", min_exact=0.98)
        elif i == 0:  # v_proj reads this library's norm, which may move a bf16 rounding
            assert_close(va, ve, f"layer {i}: V pages", min_exact=0.98)
            assert_close(ka, ke, f"layer {i}: K pages", min_exact=0.98)
        else:  # deeper layers see the previous layers' differences: the logits' tolerance
            for x, y, what in ((ka, ke, "K"), (va, ve, "V")):
                err = (x.float() - y.float()).abs()
                assert (err <= ATOL + RTOL * y.float().abs()).all(), f"layer {i}: {what} pages"
        # every slot outside the written ones is still the allocator's zero
        for cache in (a.k_cache, a.v_cache):
            rest = cache.clone()
            rest[bm, :, sm, :] = 0
            assert not rest.view(torch.int16).any(), f"layer {i}: an unwritten slot changed"
