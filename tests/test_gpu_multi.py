"""Multi-GPU paths over real NCCL (skipped with fewer than 2 GPUs): the
row-split quantize of one matrix over 2 ranks equals the single-GPU quantize
bit for bit; the token/row-split GPTQ layer gives every rank the same
tensors.  Each rank is a child process on its own GPU (NVLS off)."""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu

needs_two = pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                               reason="needs 2 GPUs")


def _rank_main(rank, world, port, q):
    import datetime

    import torch.distributed as dist

    from memboost_b200 import _C, gptq, rowsplit, workloads
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        comm = rowsplit.DistComm()
        ok = {}
        for name, case in (("single_4096", workloads.single_4096()),
                           ("shifted", workloads.small_case(2048, 1040, 12, "shifted"))):
            w, h = case.weights.cuda(), case.hessian_diag.cuda()
            r0, r1 = rowsplit.slab_bounds(w.shape[0], w.shape[1], world)[rank]
            res = rowsplit.quantize_rows(w[r0:r1].contiguous(), w.shape[0], w.shape[1],
                                         case.ratio_4bit, h, comm)
            # every rank's slab tensors, gathered in rank order
            parts = [None] * world
            dist.all_gather_object(parts, [t.cpu() for t in res.tensors])
            slabs = [rowsplit.SlabResult(0, 0, p, 0, 0, 0) for p in parts]
            got = rowsplit.assemble(slabs)
            want = [t.cpu() for t in _C.quantize(w, case.ratio_4bit, h)]
            same = all(a.shape == b.shape and torch.equal(
                a.view(torch.int16) if a.dtype == torch.float16 else a,
                b.view(torch.int16) if b.dtype == torch.float16 else b) for a, b in zip(got, want))
            ok[name] = same
        weights, inputs = workloads.gptq_layer(tokens=4096, device="cuda", scale=8)
        local = {k: x[rank::world].contiguous() for k, x in inputs.items()}
        lq = gptq.quantize_layer_distributed(weights, local, comm, 0.1)
        p2 = [None] * world
        dist.all_gather_object(p2, {n: t.packed_2bit.cpu() for n, t in lq.items()})
        ok["gptq_same_on_ranks"] = all(torch.equal(p2[0][n], p2[r][n]) for r in range(world)
                                       for n in p2[0])
        q_put = (rank, ok)
    except Exception as e:  # reported to the test
        q_put = (rank, {"error": repr(e)[:300]})
    finally:
        dist.destroy_process_group()
    q.put(q_put)


@needs_two
def test_rowsplit_and_gptq_over_nccl():
    import multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    import queue
    import time
    res = {}
    t_end = time.monotonic() + 300
    while len(res) < len(procs) and time.monotonic() < t_end:
        try:
            r, ok = q.get(timeout=2)
            res[r] = ok
        except queue.Empty:
            # a rank that died without reporting ends the test at once
            dead = [p.exitcode for p in procs if p.exitcode not in (None, 0)]
            assert not dead, f"a rank exited with {dead}"
    for p in procs:
        p.join(60)
        if p.is_alive():
            p.kill()
    assert len(res) == len(procs), "ranks did not report within 300 s"
    for r in range(2):
        assert "error" not in res[r], res[r]
        assert all(res[r].values()), res[r]
