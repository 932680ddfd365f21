"""Token sharding and the validation all-gather on CPU ranks (gloo, world
size 2): each rank runs its shard of the path's row-wise ops through the CPU
oracle, the shards are gathered, and rank 0 checks the result equals the
unsharded computation bit for bit (rows are independent, so sharding must not
change a single bit).  Covers uneven and empty shards."""

import os
import socket
import sys

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tinyserver_b200.sharding import gather_rows, shard_range, shard_rows

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_shard_ranges_tile_the_batch():
    for T in (0, 1, 7, 8192, 65536):
        for P in (1, 2, 3, 4, 8):
            spans = [shard_range(T, P, r) for r in range(P)]
            assert spans[0][0] == 0 and spans[-1][1] == T
            assert all(spans[i][1] == spans[i + 1][0] for i in range(P - 1))
            sizes = [e - s for s, e in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_range(8, 2, 2)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, T: int, result_q) -> None:
    sys.path.insert(0, ROOT)
    from datetime import timedelta

    from oracle import oracle

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        g = torch.Generator().manual_seed(11)
        H = 256
        x = torch.randn(T, H, generator=g).to(torch.bfloat16)
        res = torch.randn(T, H, generator=g).to(torch.bfloat16)
        w = (1 + 0.02 * torch.randn(H, generator=g)).to(torch.bfloat16)
        gate = torch.randn(T, 64, generator=g).to(torch.bfloat16)
        up = torch.randn(T, 64, generator=g).to(torch.bfloat16)
        y, h = oracle.add_rmsnorm(shard_rows(x, world, rank), shard_rows(res, world, rank), w,
                                  1e-6)
        act = oracle.silu_and_mul(shard_rows(gate, world, rank), shard_rows(up, world, rank))
        ys, hs, acts = gather_rows(y), gather_rows(h), gather_rows(act)
        if rank == 0:
            ey, eh = oracle.add_rmsnorm(x, res, w, 1e-6)
            ok = (torch.equal(ys, ey) and torch.equal(hs, eh)
                  and torch.equal(acts, oracle.silu_and_mul(gate, up)))
            result_q.put(("ok" if ok else "mismatch", T))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("T", [1, 7, 300])
def test_gloo_two_ranks_gather_equals_unsharded(T):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, T, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    assert codes == [0, 0], codes
    assert q.get(timeout=5) == ("ok", T)
