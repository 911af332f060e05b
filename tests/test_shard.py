"""Multi-rank host logic on CPU: two gloo ranks split a set of matrices by
LPT, quantize their shares (the CPU oracle stands in for the GPU kernels,
which these ranks do not have), gather the results and agree on the maximum
of their timings; the union equals a single-process run."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from memboost_b200 import shard


def test_lpt_partition_covers_and_balances():
    costs = [7, 3, 9, 1, 4, 4, 8, 2]
    parts = shard.lpt_partition(costs, 3)
    flat = sorted(i for p in parts for i in p)
    assert flat == list(range(len(costs)))
    loads = [sum(costs[i] for i in p) for p in parts]
    assert max(loads) - min(loads) <= max(costs)
    assert shard.lpt_partition(costs, 1) == [list(range(len(costs)))]
    assert shard.lpt_partition([], 2) == [[], []]
    with pytest.raises(ValueError):
        shard.lpt_partition(costs, 0)


def _cases():
    rng = np.random.default_rng(3)
    shapes = [(48, 64), (16, 128), (33, 80), (64, 32), (8, 256), (40, 48), (24, 96)]
    out = []
    for M, K in shapes:
        w = (rng.standard_normal((M, K)) * 0.02).astype(np.float16)
        h = np.exp(rng.standard_normal(K)).astype(np.float32)
        out.append((w, h))
    return out


def _quantize(case):
    from oracle import oracle
    w, h = case
    return oracle.quantize(w, 0.25, h)


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime

    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        cases = _cases()
        local = shard.quantize_shard(cases, rank, world, lambda c: c[0].size, _quantize)
        allres = shard.gather_to_all(local)
        t = shard.max_over_ranks(float(rank + 1) * 1.5)
        q.put((rank, sorted(local), sorted(allres), t,
               {i: {k: np.asarray(v) for k, v in r.items()} for i, r in allres.items()}
               if rank == 0 else None))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_gloo_ranks_shard_and_gather():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    got.sort(key=lambda x: x[0])
    n = len(_cases())
    local0, local1 = got[0][1], got[1][1]
    assert sorted(local0 + local1) == list(range(n)) and not set(local0) & set(local1)
    assert got[0][2] == got[1][2] == list(range(n))
    assert got[0][3] == got[1][3] == 3.0
    single = {i: _quantize(c) for i, c in enumerate(_cases())}
    for i in range(n):
        for k, v in single[i].items():
            assert np.array_equal(np.asarray(v), got[0][4][i][k]), (i, k)


def test_single_process_fallbacks():
    assert shard.max_over_ranks(2.5) == 2.5
    assert shard.gather_to_all({1: "a"}) == {1: "a"}
    assert torch.distributed.is_available()
