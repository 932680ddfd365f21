"""Shared test helpers: fixture loading, tolerances, mapping builders.

Tolerances are the parity contract of the path:

* embedding gather and KV-cache slot placement: bit-exact;
* RMSNorm / RoPE / SiLU-and-mul outputs in bf16 or fp16: |a - e| <= 2e-2 + 1e-2 * |e|
  (fp32 accumulation inside the kernels);
* the same ops in fp32: |a - e| <= 1e-5 + 1e-5 * |e|.
"""

from __future__ import annotations

import os

import torch

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

BF16_ATOL, BF16_RTOL = 2e-2, 1e-2
F32_ATOL, F32_RTOL = 1e-5, 1e-5


def load_golden(name: str) -> dict:
    return torch.load(os.path.join(GOLDEN, name), weights_only=False, map_location="cpu")


def tol(dtype: torch.dtype) -> tuple[float, float]:
    if dtype == torch.float32:
        return F32_ATOL, F32_RTOL
    return BF16_ATOL, BF16_RTOL


def assert_close(actual: torch.Tensor, expected: torch.Tensor, what: str = "",
                 min_exact: float | None = None) -> None:
    """Tolerance check of the parity contract; for 16-bit dtypes optionally also
    require that a fraction ``min_exact`` of the elements match bit for bit (in
    fp32 the order of a reduction already moves the last bit, so there the
    tolerance alone applies)."""
    actual = actual.detach().cpu()
    expected = expected.detach().cpu()
    assert actual.shape == expected.shape, (what, actual.shape, expected.shape)
    assert actual.dtype == expected.dtype, (what, actual.dtype, expected.dtype)
    atol, rtol = tol(expected.dtype)
    a = actual.float()
    e = expected.float()
    assert torch.isfinite(a).all(), f"{what}: non-finite output"
    err = (a - e).abs()
    bound = atol + rtol * e.abs()
    bad = err > bound
    if bad.any():
        i = int(bad.flatten().nonzero()[0])
        raise AssertionError(
            f"{what}: {int(bad.sum())} of {bad.numel()} elements outside tolerance; "
            f"max abs err {float(err.max()):.3g}; first at flat {i}: "
            f"{float(a.flatten()[i])} vs {float(e.flatten()[i])}")
    if min_exact is not None and expected.dtype != torch.float32:
        exact = (actual.view(-1) == expected.view(-1)).float().mean().item()
        assert exact >= min_exact, f"{what}: only {exact:.4%} bit-exact (need {min_exact:.2%})"


def prefill_mapping(seq_lens: list[int], block_tables: list[list[int]], block_size: int,
                    start_positions: list[int] | None = None,
                    dtype: torch.dtype = torch.int64) -> tuple[torch.Tensor, torch.Tensor]:
    """block/slot mapping per token, the way server/model/patches/qwen3.py:296-310
    (prefill from position 0) and tests/model/test_kv_cache_kernels.py:16-37
    (any start position) build it."""
    starts = start_positions or [0] * len(seq_lens)
    bm, sm = [], []
    for n, bt, p0 in zip(seq_lens, block_tables, starts):
        for j in range(n):
            p = p0 + j
            bm.append(bt[p // block_size])
            sm.append(p % block_size)
    return torch.tensor(bm, dtype=dtype), torch.tensor(sm, dtype=dtype)


def expected_pool(before: torch.Tensor, written: list, rows: torch.Tensor) -> torch.Tensor:
    """Rebuild a (2, 1, N, Hkv, B, D) pool from its prior contents and the rows
    (len(written), 2, Hkv, D) the reference wrote at ``written`` (block, slot) pairs."""
    out = before.clone()
    for i, (b, s) in enumerate(written):
        out[:, 0, b, :, s, :] = rows[i]
    return out


def snapshot_pool(pool: torch.Tensor) -> torch.Tensor:
    """A copy of a (2, L, N, Hkv, B, D) pool to check unwritten slots against
    (same device; a c5-sized 26 GB pool fits beside its copy on a B200)."""
    return pool.clone()


def assert_untouched(pool: torch.Tensor, snapshot: torch.Tensor, block_mapping: torch.Tensor,
                     slot_mapping: torch.Tensor, layer: int = 0, chunk_blocks: int = 8192) -> None:
    """Every pool element outside the rows (block_mapping[t], :, slot_mapping[t])
    of ``layer`` equals ``snapshot`` bit for bit (compared as integers, so NaN
    poison compares too).  ``snapshot`` is consumed: the written rows are
    copied into it from the pool (their contents are checked elsewhere), then
    the two are compared chunk by chunk along the block dimension."""
    snapshot[:, layer, block_mapping, :, slot_mapping, :] = \
        pool[:, layer, block_mapping, :, slot_mapping, :]
    as_int = {2: torch.int16, 4: torch.int32, 1: torch.int8, 8: torch.int64}[pool.element_size()]
    n = pool.shape[2]
    for b0 in range(0, n, chunk_blocks):
        a = pool[:, :, b0:b0 + chunk_blocks].contiguous().view(as_int)
        e = snapshot[:, :, b0:b0 + chunk_blocks].contiguous().view(as_int)
        if not torch.equal(a, e):
            diff = (a != e).nonzero()[0].tolist()
            diff[2] += b0
            raise AssertionError(f"an unwritten cache element changed, first at pool index {diff}")


def reference_module(name: str):
    """Import a module of the reference itself (e.g. ``server.model.patches.qwen3``)
    from its offline install in baseline/_ref, or the directory TINYSERVER_REF
    names; the calling test is skipped, with the reason, when neither holds it."""
    import pytest

    from baseline.reference_gpu import load

    try:
        return load(name)
    except ImportError as e:
        pytest.skip(f"the reference is not importable here: {e}")
