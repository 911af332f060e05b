"""GPTQ calibration feeding memboost's mixed 2/4-bit format, on B200.

The GPTQ steps of the reference's ``models/llama.py`` with the same names and
argument meaning:

* ``hessian`` / ``HessianAccumulator`` -- H = X^T X accumulated in fp32 and
  divided by the token count (llama.py:523-528, 547-551), on the tcgen05
  tensor-core kernel of ``csrc/hessian.cu``;
* ``gptq_inverse`` -- damping, Cholesky, inverse, upper Cholesky of H^-1
  (llama.py:177-203), torch.linalg as in the reference;
* ``compute_group_precision`` -- torch sensitivity sum + top-k
  (llama.py:209-231), the reference's own tensor expression;
* ``gptq_quantize`` -- the blockwise error-propagating rounding
  (llama.py:234-294) on the kernel of ``csrc/gptq.cu``, bit-identical to the
  reference;
* ``make_quantized_linear`` / ``QuantizedLinear`` -- GPTQ then
  ``memboost.quantize`` with the forced hessian that makes it select the same
  4-bit groups (llama.py:331-371, 91-105);
* ``quantize_layer`` -- the per-layer sequence of llama.py:530-617 (4
  Hessians, 4 inverses, 7 GPTQ + quantize calls) on given calibration inputs.
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _C
from .formats import GROUP_SIZE_1ST, QuantizedTensor
from .ops import dequantize, quantize

GROUP_SIZE = GROUP_SIZE_1ST
GPTQ_DIV_TRUE = _C.GPTQ_DIV_TRUE
GPTQ_DIV_RECIPROCAL = _C.GPTQ_DIV_RECIPROCAL


def hessian(x: torch.Tensor, alpha: float = 1.0, out: torch.Tensor | None = None,
            accumulate: bool = False, status: torch.Tensor | None = None) -> torch.Tensor:
    """alpha * x^T x (or out += alpha * x^T x) for x [tokens, K] fp16/bf16."""
    return _C.hessian(x, alpha=alpha, out=out, accumulate=accumulate, status=status)


class HessianAccumulator:
    """Running H = sum of x^T x over calibration batches, then H / tokens.

    ``add`` is the reference's forward hook (llama.py:523-528: x viewed as
    [-1, K], H += x^T x in fp32); ``finalize`` its normalisation
    (llama.py:547-551: H.div_(total_tokens))."""

    def __init__(self, K: int, device=None):
        device = torch.device("cuda", torch.cuda.current_device()) if device is None \
            else torch.device(device)
        self.K = K
        self.H = torch.zeros((K, K), dtype=torch.float32, device=device)
        self.status = torch.zeros(1, dtype=torch.int32, device=device)
        self.tokens = 0

    def add(self, x: torch.Tensor) -> None:
        x = x.detach().reshape(-1, x.shape[-1])
        if x.shape[1] != self.K:
            raise RuntimeError(f"expected {self.K} features, got {x.shape[1]}")
        hessian(x, out=self.H, accumulate=True, status=self.status)
        self.tokens += int(x.shape[0])

    def finalize(self, total_tokens: int | None = None) -> torch.Tensor:
        if int(self.status.item()) != 0:
            raise RuntimeError("hessian kernel reported a pipeline timeout")
        self.H.div_(self.tokens if total_tokens is None else total_tokens)
        return self.H


def gptq_inverse(H: torch.Tensor):
    """(h_diag, Hinv_cho) of llama.py:177-203; damps H in place as the
    reference does: damp = max(0.01 * max|diag H|, 1e-6) added to the
    diagonal, diagonal entries below 1e-8 set to 1, then Cholesky inverse,
    h_diag = diag(H^-1), and the upper Cholesky factor of H^-1 + 1e-8 I."""
    d = H.diagonal()
    damp = max((0.01 * d.abs().max()).item(), 1e-6)
    d.add_(damp)
    dead = d < 1e-8
    if dead.any():
        d[dead] = 1.0
    Hinv = torch.cholesky_inverse(torch.linalg.cholesky(H))
    h_diag = Hinv.diag().clone()
    Hinv.diagonal().add_(1e-8)
    return h_diag, torch.linalg.cholesky(Hinv, upper=True)


def compute_group_precision(W: torch.Tensor, h_diag: torch.Tensor, ratio_4bit: float):
    """uint8 [K // 16]: 1 for the int(ratio * groups) groups of largest
    sum_{rows, cols in group} w^2 / clamp(h_diag, 1e-8) (llama.py:209-231,
    the same torch expression, so the same sums and top-k)."""
    M, K = W.shape
    ng = K // GROUP_SIZE
    inv_h = 1.0 / h_diag.clamp(min=1e-8)
    sens = (W.pow(2) * inv_h.unsqueeze(0)).view(M, ng, GROUP_SIZE).sum(dim=(0, 2))
    n4 = int(ratio_4bit * ng)
    gp = torch.zeros(ng, dtype=torch.uint8, device=W.device)
    if n4 > 0:
        gp[sens.topk(n4).indices] = 1
    return gp


def gptq_quantize(W: torch.Tensor, Hinv_cho: torch.Tensor, group_precision: torch.Tensor,
                  blocksize: int = 128, scalar_division: int | None = None,
                  rows: tuple | None = None) -> torch.Tensor:
    """Q of llama.py:234-294 (fp32 [M, K]), bit-identical to the reference.

    ``scalar_division`` picks which run of the reference to reproduce:
    GPTQ_DIV_RECIPROCAL (default) -- tensors on a CUDA device, where PyTorch
    divides by the Python-float scale as a multiplication by its fp32
    reciprocal; GPTQ_DIV_TRUE -- tensors on the CPU (IEEE quotient)."""
    if scalar_division is None:
        scalar_division = GPTQ_DIV_RECIPROCAL
    return _C.gptq_quantize(W, Hinv_cho, group_precision, blocksize=blocksize,
                            scalar_division=scalar_division, rows=rows)


def forced_hessian_diag(group_precision: torch.Tensor, K: int, device=None) -> torch.Tensor:
    """The hessian_diag of llama.py:356-364 that makes memboost's selection
    pick exactly the groups marked in ``group_precision``: 1e-10 on 4-bit
    groups, 1e10 on 2-bit groups, 1.0 past the last whole group."""
    device = group_precision.device if device is None else device
    h = torch.ones(K, dtype=torch.float32, device=device)
    ng = K // GROUP_SIZE
    four = group_precision[:ng].to(device=device).repeat_interleave(GROUP_SIZE) == 1
    h[:ng * GROUP_SIZE] = torch.where(four, torch.tensor(1e-10, device=device),
                                      torch.tensor(1e10, device=device))
    return h


class QuantizedLinear(nn.Module):
    """Linear layer over a memboost QuantizedTensor (llama.py:91-105):
    forward = F.linear(x.half(), dequantize(q_weight))."""

    def __init__(self, in_features: int, out_features: int):
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        self.q_weight: QuantizedTensor | None = None

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return F.linear(x.to(torch.float16), dequantize(self.q_weight))


def make_quantized_linear(W_fp32: torch.Tensor, h_diag: torch.Tensor, Hinv_cho: torch.Tensor,
                          ratio_4bit: float, blocksize: int = 128) -> QuantizedLinear:
    """GPTQ + memboost quantize of one weight matrix (llama.py:331-371)."""
    M, K = W_fp32.shape
    if ratio_4bit <= 0:
        gp = torch.zeros(K // GROUP_SIZE, dtype=torch.uint8, device=W_fp32.device)
        Q = gptq_quantize(W_fp32, Hinv_cho, gp, blocksize=blocksize)
        qt = quantize(Q.to(torch.float16).contiguous(), ratio_4bit=0.0)
    else:
        gp = compute_group_precision(W_fp32, h_diag, ratio_4bit)
        Q = gptq_quantize(W_fp32, Hinv_cho, gp, blocksize=blocksize)
        qt = quantize(Q.to(torch.float16).contiguous(), ratio_4bit=ratio_4bit,
                      hessian_diag=forced_hessian_diag(gp, K))
    ql = QuantizedLinear(K, M)
    ql.q_weight = qt
    return ql


# weight name -> which calibration input (Hessian) it shares (llama.py:555-593)
LAYER_INPUTS = {
    "self_attn.q_proj": "attn", "self_attn.k_proj": "attn", "self_attn.v_proj": "attn",
    "self_attn.o_proj": "o", "mlp.gate_proj": "mlp", "mlp.up_proj": "mlp",
    "mlp.down_proj": "down",
}


class InverseWorkers:
    """The layer's inverses (gptq_inverse), each in a host thread and on a
    CUDA stream of its own.  The Cholesky factorisations are the longest
    part of a layer (the 11008 x 11008 one ~105 ms of a ~200 ms layer) and
    wait on the host for their error checks (with the interpreter lock
    released), so started as soon as their Hessian is final they overlap one
    another and the caller's Hessians, GPTQ updates and quantize calls on its
    own stream.  The results are those of gptq_inverse: the same torch
    calls."""

    _linalg_ready = set()  # devices whose torch.linalg set-up ran
    _streams = {}          # device -> the workers' streams, kept across layers

    def __init__(self, device, workers: int = 4):
        from concurrent.futures import ThreadPoolExecutor
        self.device = torch.device(device)
        if self.device not in InverseWorkers._linalg_ready:
            # torch.linalg initialises its CUDA back end lazily on the first
            # call, which must not happen in several threads at once
            e = torch.eye(2, device=self.device)
            torch.linalg.cholesky(torch.cholesky_inverse(torch.linalg.cholesky(e)), upper=True)
            InverseWorkers._linalg_ready.add(self.device)
        # the same streams every layer: the caching allocator and the solver
        # keep their blocks and workspaces per stream
        pool = InverseWorkers._streams.setdefault(self.device, [])
        while len(pool) < workers:
            pool.append(torch.cuda.Stream(self.device))
        self.streams = pool[:workers]
        self.pool = ThreadPoolExecutor(max_workers=workers)
        self.futures = {}

    def start(self, key, H: torch.Tensor) -> None:
        """Begin the inverse of H (complete in stream order on the current
        stream)."""
        ready = torch.cuda.Event()
        ready.record(torch.cuda.current_stream(self.device))
        s = self.streams[len(self.futures) % len(self.streams)]
        self.futures[key] = self.pool.submit(self._run, H, ready, s)

    def _run(self, H: torch.Tensor, ready, s):
        with torch.cuda.device(self.device):
            s.wait_event(ready)
            with torch.cuda.stream(s):
                H.record_stream(s)
                h_diag, hinv_cho = gptq_inverse(H)
                done = torch.cuda.Event()
                done.record(s)
        return h_diag, hinv_cho, done

    def take(self, key):
        """(h_diag, Hinv_cho) of key, ordered before later work on the
        current stream."""
        h_diag, hinv_cho, done = self.futures[key].result()
        cur = torch.cuda.current_stream(self.device)
        cur.wait_event(done)
        h_diag.record_stream(cur)
        hinv_cho.record_stream(cur)
        return h_diag, hinv_cho

    def close(self) -> None:
        self.pool.shutdown(wait=True)


def quantize_layer(weights: dict, inputs: dict, ratio_4bit: float = 0.1,
                   blocksize: int = 128) -> dict:
    """One transformer layer's GPTQ (llama.py:530-617): the four Hessians
    from the calibration inputs (``inputs``: "attn", "o", "mlp", "down" ->
    [tokens, K] fp16/bf16), their inverses, then GPTQ + quantize of the seven
    fp32 weight matrices (``weights``: names of ``LAYER_INPUTS``).  Returns
    name -> QuantizedTensor.

    The largest Hessian goes first and every inverse runs beside the rest
    (InverseWorkers); the weights then take their turn in the order their
    inverses come ready (the small Hessians' first).  The results do not
    depend on the order."""
    dev = next(iter(inputs.values())).device
    workers = InverseWorkers(dev, workers=len(inputs))
    try:
        for key in sorted(inputs, key=lambda k: -inputs[k].shape[-1]):
            x = inputs[key]
            acc = HessianAccumulator(x.shape[-1], x.device)
            acc.add(x)
            workers.start(key, acc.finalize())
        out = {}
        for name in sorted(weights, key=lambda n: inputs[LAYER_INPUTS[n]].shape[-1]):
            h_diag, hinv_cho = workers.take(LAYER_INPUTS[name])
            out[name] = make_quantized_linear(weights[name], h_diag, hinv_cho, ratio_4bit,
                                              blocksize=blocksize).q_weight
    finally:
        workers.close()
    return {name: out[name] for name in weights}


def even_rows(M: int, world: int) -> list[tuple[int, int]]:
    """Contiguous, as-even-as-possible row ranges of M rows over `world` ranks."""
    return [(M * r // world, M * (r + 1) // world) for r in range(world)]


def quantize_layer_distributed(weights: dict, inputs_local: dict, comm, ratio_4bit: float = 0.1,
                               blocksize: int = 128, inverses: dict | None = None) -> dict:
    """One layer's GPTQ (llama.py:530-617) with the calibration tokens and the
    weight rows split over ranks; every rank ends with the same
    QuantizedTensors.

    * Hessians: each rank accumulates x^T x over its own tokens
      (``inputs_local``: key -> [tokens_r, K]) on the tcgen05 kernel; the
      partial sums are all-reduced (NCCL) and divided by the total token count
      (llama.py:523-528, 547-551).
    * Inverses: the four damped Cholesky inverses (llama.py:177-203) run on
      different ranks (key i on rank i mod world) and are broadcast.
    * GPTQ: each rank updates its rows of every weight (mb_gptq_quantize_rows,
      group parameters over all rows), the fp16 rows are all-gathered, and the
      memboost quantize (llama.py:331-371) runs on the whole Q.
    Given the same inverses (``inverses``: key -> (h_diag, Hinv_cho)) the
    result equals quantize_layer's bit for bit; the all-reduced Hessians
    differ from one device's accumulation only by fp32 summation order.
    ``comm``: rowsplit.DistComm or rowsplit.LocalComm."""
    if inverses is None:
        inverses = {}
        keys = list(inputs_local)
        dev = next(iter(inputs_local.values())).device
        tok = torch.tensor([float(sum(int(x.reshape(-1, x.shape[-1]).shape[0])
                                      for x in inputs_local.values()) / max(1, len(keys)))],
                           dtype=torch.float64, device=dev)
        total = float(comm.all_reduce_sum(tok).item())
        for i, key in enumerate(keys):
            x = inputs_local[key].reshape(-1, inputs_local[key].shape[-1])
            K = int(x.shape[1])
            H = hessian(x) if x.shape[0] > 0 else torch.zeros((K, K), device=x.device)
            H = comm.all_reduce_sum(H)
            H.div_(total)
            owner = i % comm.world
            if comm.rank == owner:
                h_diag, hc = gptq_inverse(H)
            else:
                h_diag = torch.empty((K,), dtype=torch.float32, device=x.device)
                hc = torch.empty((K, K), dtype=torch.float32, device=x.device)
            del H
            inverses[key] = (comm.broadcast(h_diag, owner), comm.broadcast(hc, owner))
    out = {}
    for name, W in weights.items():
        h_diag, hc = inverses[LAYER_INPUTS[name]]
        M, K = W.shape
        if ratio_4bit > 0:
            gp = compute_group_precision(W, h_diag, ratio_4bit)
        else:
            gp = torch.zeros(K // GROUP_SIZE, dtype=torch.uint8, device=W.device)
        r0, r1 = even_rows(M, comm.world)[comm.rank]
        Qs = gptq_quantize(W, hc, gp, blocksize=blocksize, rows=(r0, r1))
        Q = comm.all_gather_rows(Qs.to(torch.float16)).contiguous()
        if ratio_4bit > 0:
            out[name] = quantize(Q, ratio_4bit=ratio_4bit, hessian_diag=forced_hessian_diag(gp, K))
        else:
            out[name] = quantize(Q, ratio_4bit=0.0)
    return out
