"""Host logic of the row-split quantize, on CPU: slab bounds (2nd-order
period granularity, coverage), strip columns and ratio, CSR row-pointer
offsets, and the exchanges through torch.distributed with two gloo ranks
(equal and uneven row counts, rank order)."""
import math
import os

import pytest
import torch

from memboost_b200 import rowsplit


@pytest.mark.parametrize("M,K,world", [(28672, 8192, 8), (8192, 28672, 8), (4096, 11008, 3),
                                       (4096, 4096, 2), (17, 100, 2), (1000, 4104, 7),
                                       (11008, 4096, 5)])
def test_slab_bounds(M, K, world):
    b = rowsplit.slab_bounds(M, K, world)
    assert len(b) == world and b[0][0] == 0 and b[-1][1] == M
    gran = rowsplit.slab_granularity(K)
    ng = (K + 15) // 16
    assert gran == 256 // math.gcd(ng, 256)
    for (r0, r1), (s0, _) in zip(b, b[1:]):
        assert r1 == s0 and r1 % gran == 0
        assert (r1 * ng) % 256 == 0  # no 2nd-order chunk spans two slabs
    sizes = [r1 - r0 for r0, r1 in b]
    assert max(sizes) - min(sizes) <= gran + (M % gran)


def test_strip_helpers():
    assert rowsplit.pending_strip_columns([0, 2], 40) == list(range(16)) + list(range(32, 40))
    for n in range(1, 200):
        for need in range(1, n):
            r = rowsplit.strip_ratio(need, n)
            assert int(r * n) == need
    assert rowsplit.row_ptr_offsets([3, 0, 5, 1]) == [0, 3, 3, 8]


def _worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        comm = rowsplit.DistComm()
        parts = comm.all_gather(torch.full((4,), rank, dtype=torch.uint8))
        ok1 = [int(p[0]) for p in parts] == list(range(world))
        rows = torch.arange(rank * 10, rank * 10 + 3 + rank, dtype=torch.float16).view(-1, 1)
        cat = comm.all_gather_rows(rows.expand(-1, 2).contiguous())
        want = torch.cat([torch.arange(r * 10, r * 10 + 3 + r, dtype=torch.float16)
                          for r in range(world)]).view(-1, 1).expand(-1, 2)
        ok2 = torch.equal(cat, want)
        nnz = comm.all_gather(torch.tensor([5 * rank + 1]))
        ok3 = rowsplit.row_ptr_offsets([int(x) for x in nnz]) == [0, 1][:world]
        q.put((rank, ok1, ok2, ok3))
    finally:
        dist.destroy_process_group()


def test_gloo_two_rank_exchanges():
    import multiprocessing as mp
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    res = sorted(q.get(timeout=5) for _ in procs)
    assert [r[0] for r in res] == [0, 1]
    assert all(all(r[1:]) for r in res), res
