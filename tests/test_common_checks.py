"""The untouched-slot check itself, on CPU tensors: it must catch any change
outside the written rows, including two changes that cancel in a sum."""

import pytest
import torch

from tests.common import assert_untouched, snapshot_pool


def _pool_and_rows():
    g = torch.Generator().manual_seed(3)
    pool = torch.randn(2, 1, 40, 2, 16, 8, generator=g).to(torch.bfloat16)
    bm = torch.tensor([3, 3, 17, 39])
    sm = torch.tensor([0, 5, 15, 7])
    return pool, bm, sm


def test_written_rows_only_pass():
    pool, bm, sm = _pool_and_rows()
    snap = snapshot_pool(pool)
    pool[:, 0, bm, :, sm, :] = torch.ones(4, 2, 2, 8, dtype=pool.dtype)
    assert_untouched(pool, snap, bm, sm, chunk_blocks=7)


def test_compensating_changes_are_caught():
    pool, bm, sm = _pool_and_rows()
    snap = snapshot_pool(pool)
    as_int = pool.view(torch.int16)
    as_int[0, 0, 5, 1, 2, 3] += 1   # outside the written rows
    as_int[1, 0, 20, 0, 9, 0] -= 1  # cancels the first in an additive checksum
    with pytest.raises(AssertionError, match="unwritten cache element changed"):
        assert_untouched(pool, snap, bm, sm, chunk_blocks=7)


def test_nan_poison_compares_exactly():
    pool, bm, sm = _pool_and_rows()
    pool[0, 0, 9] = float("nan")
    snap = snapshot_pool(pool)
    assert_untouched(pool, snap, bm, sm)
