"""Row-split quantize: one weight matrix's rows over several GPUs.

memboost's quantize (core/torch_ops.cu:105-264) couples every row of a
matrix: each 16-column group's min / max runs over all rows
(core/quantize.cu:103-128), its sensitivity is one serial fp32 sum over all
rows (quantize.cu:72-98) and the 4-bit groups are the global top-k of those
sums (torch_ops.cu:149-179).  To quantize a matrix too large for one GPU's
time budget (the Llama-70B-shaped MLP matrices, 28672 x 8192), each rank
takes a contiguous slab of rows and the ranks exchange what couples them:

1. every rank streams its slab once and keeps, per group, a 32-byte record
   (min, max, the prediction and moment of its sensitivity terms, rows);
2. one all-gather of the records (ng x 32 bytes per rank, NCCL over NVLink);
3. every rank combines the records in row order into the same group
   parameters and the same rigorous sensitivity intervals a single pass
   would give, and takes the same selection;
4. groups whose interval straddles the 4-bit boundary (a few at most) need
   their exact serial sums: their 16-column strips are all-gathered (M x 16
   fp16 per group) and quantized as one small matrix on every rank, which
   settles them exactly as the single-GPU selection does;
5. every rank encodes its slab; the outlier counts are all-gathered to offset
   the slabs' CSR row pointers.

Slab boundaries are multiples of 256 / gcd(ng, 256) rows so that no 2nd-order
chunk of 256 flattened scales spans two ranks.  The result equals
memboost_b200.quantize on the whole matrix bit for bit.

``Comm`` is the exchange: ``DistComm`` uses torch.distributed (NCCL for GPUs,
gloo for CPU tests); ``quantize_rows_local`` runs all ranks' slabs in one
process with the exchanges done in memory.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from . import _C
from .formats import GROUP_SIZE_1ST, GROUP_SIZE_2ND

RECORD_BYTES = 32


def slab_granularity(K: int) -> int:
    """Rows per 2nd-order period: slab boundaries must be multiples of it."""
    ng = (K + GROUP_SIZE_1ST - 1) // GROUP_SIZE_1ST
    return GROUP_SIZE_2ND // math.gcd(ng, GROUP_SIZE_2ND)


def slab_bounds(M: int, K: int, world: int) -> list[tuple[int, int]]:
    """Contiguous row ranges [r0, r1) per rank, as even as the granularity
    allows, boundaries multiples of slab_granularity(K) (the last slab takes
    the remainder; a rank may get an empty slab only when M is tiny)."""
    if world < 1:
        raise ValueError("world must be >= 1")
    gran = slab_granularity(K)
    units = (M + gran - 1) // gran
    bounds, start = [], 0
    for p in range(world):
        end_u = (units * (p + 1)) // world
        end = min(M, end_u * gran)
        bounds.append((start, end))
        start = end
    return bounds


def row_ptr_offsets(nnz_per_rank: list[int]) -> list[int]:
    """Exclusive prefix of the ranks' outlier counts: each slab's CSR row
    pointers plus its offset are the whole matrix's."""
    out, acc = [], 0
    for n in nnz_per_rank:
        out.append(acc)
        acc += int(n)
    return out


def pending_strip_columns(groups: list[int], K: int) -> list[int]:
    """Columns of the given groups in order (the strip matrix): 16 per group,
    fewer for a last group past K."""
    cols = []
    for g in groups:
        cols.extend(range(g * GROUP_SIZE_1ST, min((g + 1) * GROUP_SIZE_1ST, K)))
    return cols


def strip_ratio(need: int, n_pending: int) -> float:
    """ratio_4bit for the strip matrix such that int(ratio * n_pending) ==
    need, the number of pending groups that are 4-bit."""
    r = (need + 0.5) / n_pending
    assert int(r * n_pending) == need
    return r


class DistComm:
    """Exchanges through torch.distributed (every rank calls each method in
    the same order)."""

    def __init__(self, group=None):
        import torch.distributed as dist
        self.dist = dist
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)

    def _dev(self, t: torch.Tensor) -> torch.Tensor:
        backend = self.dist.get_backend(self.group)
        return t if (backend == "nccl") == t.is_cuda else \
            t.to("cuda" if backend == "nccl" else "cpu")

    def all_gather(self, t: torch.Tensor) -> list[torch.Tensor]:
        """Equal-shaped tensors of all ranks, in rank order, on t's device."""
        x = self._dev(t.contiguous())
        parts = [torch.empty_like(x) for _ in range(self.world)]
        self.dist.all_gather(parts, x, group=self.group)
        return [p.to(t.device) for p in parts]

    def all_gather_rows(self, t: torch.Tensor) -> torch.Tensor:
        """Row-concatenation of every rank's [rows_p, ...] tensor (rows may
        differ), in rank order."""
        n = torch.tensor([t.shape[0]], dtype=torch.int64, device=t.device)
        rows = [int(x.item()) for x in self.all_gather(n)]
        pad = max(rows)
        buf = torch.zeros((pad,) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
        buf[:t.shape[0]] = t
        parts = self.all_gather(buf)
        return torch.cat([p[:r] for p, r in zip(parts, rows)], 0)


    def all_reduce_sum(self, t: torch.Tensor) -> torch.Tensor:
        """Elementwise sum over ranks (in place on a copy; t's device)."""
        x = self._dev(t.contiguous()).clone()
        self.dist.all_reduce(x, op=self.dist.ReduceOp.SUM, group=self.group)
        return x.to(t.device)

    def broadcast(self, t: torch.Tensor, src: int) -> torch.Tensor:
        """Rank src's tensor on every rank (t gives the shape and dtype)."""
        x = self._dev(t.contiguous()).clone()
        self.dist.broadcast(x, src=src, group=self.group)
        return x.to(t.device)


class LocalHub:
    """The meeting point of LocalComm ranks: threads of one process, each
    driving one emulated rank (same collective order as DistComm)."""

    def __init__(self, world: int):
        import threading
        self.world = world
        self.barrier = threading.Barrier(world)
        self.slots: list = [None] * world


class LocalComm:
    """In-process exchanges between the threads of a LocalHub: SPMD code
    written against DistComm runs unchanged with all ranks in one process
    (on one GPU), which lets the multi-rank paths be checked without a
    multi-GPU machine."""

    def __init__(self, hub: LocalHub, rank: int):
        self.hub, self.rank, self.world = hub, rank, hub.world

    def _exchange(self, t):
        self.hub.slots[self.rank] = t
        self.hub.barrier.wait()
        parts = list(self.hub.slots)
        self.hub.barrier.wait()
        return parts

    def all_gather(self, t: torch.Tensor) -> list[torch.Tensor]:
        return [p.to(t.device).clone() for p in self._exchange(t.contiguous())]

    def all_gather_rows(self, t: torch.Tensor) -> torch.Tensor:
        return torch.cat([p.to(t.device) for p in self._exchange(t.contiguous())], 0)

    def all_reduce_sum(self, t: torch.Tensor) -> torch.Tensor:
        parts = self._exchange(t.contiguous())
        out = parts[0].to(t.device).clone()
        for p in parts[1:]:
            out.add_(p.to(t.device))
        return out

    def broadcast(self, t: torch.Tensor, src: int) -> torch.Tensor:
        return self._exchange(t.contiguous())[src].to(t.device).clone()


def run_local(world: int, fn, *args):
    """Runs fn(comm, rank, *args) on `world` threads with LocalComm
    exchanges; returns the results in rank order (re-raises a rank's error)."""
    import threading
    hub = LocalHub(world)
    res: list = [None] * world
    err: list = [None] * world
    dev = torch.cuda.current_device() if torch.cuda.is_available() else None

    def body(r):
        try:
            if dev is not None:
                torch.cuda.set_device(dev)
            res[r] = fn(LocalComm(hub, r), r, *args)
        except BaseException as e:  # noqa: BLE001 -- handed to the caller
            err[r] = e
            hub.barrier.abort()

    th = [threading.Thread(target=body, args=(r,)) for r in range(world)]
    for t in th:
        t.start()
    for t in th:
        t.join()
    for e in err:
        if e is not None and not isinstance(e, threading.BrokenBarrierError):
            raise e
    for e in err:
        if e is not None:
            raise e
    return res


@dataclass
class SlabResult:
    """One rank's slab of the quantized matrix (the reference's 11 fields,
    every [M, *] field holding rows [r0, r1)) and the exchange results."""
    r0: int
    r1: int
    tensors: list           # reference order; outlier_row_ptrs offset to the whole matrix
    nnz_offset: int
    n_pending: int
    need: int


class _Slab:
    """The device state of one rank's slab across the protocol's phases."""

    def __init__(self, w_slab: torch.Tensor, K: int, ratio: float, hess: torch.Tensor | None):
        self.w = w_slab.contiguous()
        self.M = int(self.w.shape[0])
        self.K = K
        self.ratio = float(ratio)
        self.h = hess if (hess is not None and hess.numel() > 0 and ratio > 0) else None
        dev = self.w.device
        self.ws = _C.QuantizeWorkspace(max(self.M, 1), K, dev)
        self.ng = (K + GROUP_SIZE_1ST - 1) // GROUP_SIZE_1ST
        self.records = torch.empty(self.ng * RECORD_BYTES, dtype=torch.uint8, device=dev)
        self.pending = torch.empty(max(self.ng, 1), dtype=torch.int32, device=dev)
        self.counts = torch.empty(2, dtype=torch.int32, device=dev)

    def _h(self):
        return (None, 0) if self.h is None else (_C._ptr(self.h), self.h.numel())

    def stats(self) -> torch.Tensor:
        hp, hn = self._h()
        with torch.cuda.device(self.w.device):
            _C._check(_C._lib.mb_rows_stats(_C._ptr(self.w), self.M, self.K, self.ratio, hp, hn,
                                            _C._ptr(self.records), _C._ptr(self.ws.buf),
                                            self.ws.nbytes, _C._stream(self.w.device)))
        return self.records

    def select(self, records_all: torch.Tensor, n_ranks: int, M_total: int) -> tuple[list, int]:
        hp, hn = self._h()
        with torch.cuda.device(self.w.device):
            _C._check(_C._lib.mb_rows_select(
                _C._ptr(records_all), n_ranks, M_total, _C._ptr(self.w), self.M, self.K,
                self.ratio, hp, hn, _C._ptr(self.ws.buf), self.ws.nbytes, _C._ptr(self.pending),
                _C._ptr(self.counts), _C._stream(self.w.device)))
        c = self.counts.tolist()
        return self.pending[:c[0]].tolist(), int(c[1])

    def set_precision(self, groups: list, prec: torch.Tensor) -> None:
        dev = self.w.device
        g = torch.tensor(groups, dtype=torch.int32, device=dev)
        p = prec.to(device=dev, dtype=torch.uint8).contiguous()
        with torch.cuda.device(dev):
            _C._check(_C._lib.mb_rows_set_precision(_C._ptr(self.ws.buf), self.ws.nbytes, self.M,
                                                    self.K, _C._ptr(g), _C._ptr(p), len(groups),
                                                    _C._stream(dev)))

    def encode(self) -> list:
        M, K, ng = self.M, self.K, self.ng
        dev = self.w.device
        ng2 = (M * ng + GROUP_SIZE_2ND - 1) // GROUP_SIZE_2ND
        e = lambda shape, dt: torch.empty(shape, dtype=dt, device=dev)  # noqa: E731
        out = [e((M, ng), torch.int32), e((M, 2 * ng), torch.int32), e((M, ng), torch.float16),
               e((M, ng), torch.int8), e((ng2,), torch.float16), e((ng2,), torch.int8),
               e((M, ng), torch.uint8), e((ng,), torch.uint8)]
        row_ptrs = e((M + 1,), torch.int32)
        hp, hn = self._h()
        with torch.cuda.device(dev):
            _C._check(_C._lib.mb_rows_encode(
                _C._ptr(self.w), M, K, self.ratio, hp, hn, *(_C._ptr(t) for t in out),
                _C._ptr(row_ptrs), _C._ptr(self.ws.nnz), _C._ptr(self.ws.buf), self.ws.nbytes,
                _C._stream(dev)))
            nnz = int(self.ws.nnz.item())
            vals = e((nnz,), torch.float16)
            cols = e((nnz,), torch.int32)
            if nnz > 0:
                _C._check(_C._lib.mb_quantize_extract_outliers(
                    _C._ptr(self.w), M, K, _C._ptr(row_ptrs), _C._ptr(vals), _C._ptr(cols),
                    _C._ptr(self.ws.buf), self.ws.nbytes, _C._stream(dev)))
        return [*out, vals, cols, row_ptrs]


def _settle_pending(strip: torch.Tensor, h: torch.Tensor | None, groups: list, need: int,
                    K: int) -> torch.Tensor:
    """Precision (uint8 per pending group) from the exact serial sums over
    all rows: the strip matrix of the pending groups' columns quantized with
    the selection of `need` of them."""
    cols = pending_strip_columns(groups, K)
    hs = h[torch.tensor(cols, device=h.device)].contiguous()
    res = _C.quantize(strip.contiguous(), strip_ratio(need, len(groups)), hs)
    return res[7][:len(groups)]


def quantize_rows(w_slab: torch.Tensor, M_total: int, K: int, ratio_4bit: float,
                  hessian_diag: torch.Tensor | None, comm: DistComm) -> SlabResult:
    """This rank's part of the row-split quantize (every rank calls it with its
    slab of the bounds slab_bounds(M_total, K, comm.world))."""
    bounds = slab_bounds(M_total, K, comm.world)
    if any(b1 <= b0 for b0, b1 in bounds):  # every rank sees it: none enters a collective
        raise RuntimeError(f"{M_total} rows hold fewer than {comm.world} periods of "
                           f"{slab_granularity(K)} rows: some rank would get no rows")
    r0, r1 = bounds[comm.rank]
    if tuple(w_slab.shape) != (r1 - r0, K):
        raise RuntimeError(f"rank {comm.rank}: slab must be rows [{r0}, {r1}) of [{M_total}, {K}]")
    s = _Slab(w_slab, K, ratio_4bit, hessian_diag)
    recs = comm.all_gather(s.stats())
    records_all = torch.cat(recs, 0)
    groups, need = s.select(records_all, comm.world, M_total)
    if groups:
        cols = torch.tensor(pending_strip_columns(groups, K), device=s.w.device)
        strip = comm.all_gather_rows(s.w[:, cols])
        s.set_precision(groups, _settle_pending(strip, s.h, groups, need, K))
    out = s.encode()
    nnz = torch.tensor([int(out[8].numel())], dtype=torch.int64, device=s.w.device)
    offs = row_ptr_offsets([int(x.item()) for x in comm.all_gather(nnz)])
    out[10] = out[10] + offs[comm.rank]
    return SlabResult(r0, r1, out, offs[comm.rank], len(groups), need)


def quantize_rows_local(W: torch.Tensor, world: int, ratio_4bit: float,
                        hessian_diag: torch.Tensor | None) -> list[SlabResult]:
    """All ranks of the row split in this process, on W's device: the same
    phases and exchanges as quantize_rows, the collectives done in memory."""
    M, K = int(W.shape[0]), int(W.shape[1])
    bounds = [b for b in slab_bounds(M, K, world) if b[1] > b[0]]  # ranks without rows idle
    world = len(bounds)
    slabs = [_Slab(W[r0:r1], K, ratio_4bit, hessian_diag) for r0, r1 in bounds]
    records_all = torch.cat([s.stats() for s in slabs], 0)
    sel = [s.select(records_all, world, M) for s in slabs]
    groups, need = sel[0]
    assert all(x == sel[0] for x in sel), "ranks disagree on the selection"
    if groups:
        cols = torch.tensor(pending_strip_columns(groups, K), device=W.device)
        strip = torch.cat([s.w[:, cols] for s in slabs], 0)
        prec = _settle_pending(strip, slabs[0].h, groups, need, K)
        for s in slabs:
            s.set_precision(groups, prec)
    outs = [s.encode() for s in slabs]
    offs = row_ptr_offsets([int(o[8].numel()) for o in outs])
    res = []
    for (r0, r1), o, off in zip(bounds, outs, offs):
        o[10] = o[10] + off
        res.append(SlabResult(r0, r1, o, off, len(groups), need))
    return res


def assemble(slabs: list[SlabResult]) -> list:
    """The whole matrix's 11 tensors from the slabs (rank order): [M, *]
    fields and 2nd-order arrays concatenated, CSR concatenated, row pointers
    joined (each slab's last entry is the next slab's first)."""
    out = []
    for k in range(8):
        if k == 7:
            out.append(slabs[0].tensors[7])
        else:
            out.append(torch.cat([s.tensors[k] for s in slabs], 0))
    out.append(torch.cat([s.tensors[8] for s in slabs], 0))
    out.append(torch.cat([s.tensors[9] for s in slabs], 0))
    rp = [slabs[0].tensors[10][:1]] + [s.tensors[10][1:] for s in slabs]
    out.append(torch.cat(rp, 0))
    return out
