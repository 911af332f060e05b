#!/usr/bin/env python
"""Benchmark: memboost quantize throughput on B200 (FP16 GB/s quantized).

One step = quantize the whole Llama-2-7B-shaped model: 32 layers x {q, k, v,
o 4096x4096, gate / up 11008x4096, down 4096x11008}, 224 matrices, 12.95 GB
of fp16, N(0, 0.02^2) weights, lognormal(0, 1.5) hessian_diag per matrix,
ratio_4bit 0.1 -- synthetic and seeded (no checkpoint exists here), drawn on
the GPU.  At N GPUs the 224 matrices are split over the ranks by size
(longest-processing-time first, memboost_b200.shard.lpt_partition): strong
scaling, no collective on the data path; the step time is the max over
ranks.  Rank 0 prints one JSON line.

  value      device-resident throughput: every matrix of this rank's share
             quantized by one CUDA-graph replay of its launches
             (memboost_b200._C.QuantizeBatch: stats, tables, encode and the
             CSR extraction chained on the device, one launch of each kernel
             per 8 matrices, 8 graph branches); step k + 1 is enqueued
             before step k's outlier counts are read
  e2e        the public memboost_b200.quantize() call per matrix with host
             buffers: pinned H2D copies of the weights and hessians (all
             enqueued first on a copy stream), quantize, D2H of every output
             tensor, inside the timed region
  roofline   algorithmic bytes of the step's quantize calls (3.0 B per weight
             plus hessian, 2nd-order, CSR and precision bytes) / device time
             per step, against MEASURED_PEAKS.json
  cpu_baseline  the CPU oracle (C++ restatement of the reference algorithm)
             on all host cores, on row slices of the model's first layer
  sub-records (one GPU only): mlp_pair (the Llama-7B MLP pair 11008x4096 +
             4096x11008 with Student-t outliers, every plan on a stream of its
             own), single_4096 (4096x4096 quantize + dequantize, hessian
             ones), gptq_layer (one Llama-7B layer's GPTQ on 262144
             calibration tokens: s/layer and the tensor-core Hessian's
             TFLOP/s)

--impl reference times the reference algorithm on the host cores (the
oracle port, rank 0 only) on row slices of the same model, and -- as context
-- the reference's own CUDA kernels (oracle/_ref, built from its sources) on
the model's first layer, and its GPTQ layer loop restated in torch ops on
the GPU.  That arm loads nothing of memboost_b200's native library.
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import statistics
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "FP16 GB/s quantized (whole Llama-2-7B-shaped model, 224 matrices)"
UNIT = "GB/s"
WORKLOAD = ("llama2_7b model: 32 layers x {q,k,v,o 4096x4096, gate/up 11008x4096, "
            "down 4096x11008} fp16 N(0,0.02^2), 224 matrices, 12.95 GB; hessian_diag "
            "lognormal(0,1.5) per matrix; ratio_4bit 0.1; 16-col groups; matrices split over "
            "ranks by size (LPT)")

# Measured DRAM read + write (ncu, L2 kept between kernels) that the
# roofline's algorithmic bytes are compared with: one step of the whole
# model on one GPU (19.44 GB algorithmic), and one quantize call of a
# 4096x11008 / 11008x4096 matrix in the pipelined MLP-pair record (135.4 MB
# algorithmic).
TRAFFIC_PER_STEP_MODEL = 26_160_000_000
TRAFFIC_PER_CALL_MLP7B = 169_700_000


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=100)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--e2e-steps", type=int, default=2)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-sub", action="store_true", help="skip the one-GPU sub-records")
    p.add_argument("--layers", type=int, default=32, help="model layers (32 = the config)")
    p.add_argument("--per-launch", type=int, default=None,
                   help="matrices sharing one launch of each quantize kernel (1-8; default: 8, "
                        "fewer when a rank's share would make fewer launch sets than branches)")
    p.add_argument("--branches", type=int, default=8, help="parallel CUDA-graph branches")
    p.add_argument("--only", default=None,
                   choices=("mlp_pair", "single_4096", "gptq_layer", "hessian", "qgemv",
                            "rowsplit", "gptq_stream"),
                   help="run one sub-record alone and print it (small cases for profiling)")
    p.add_argument("--tokens", type=int, default=262144,
                   help="calibration tokens of the gptq_layer / hessian records")
    p.add_argument("--sub-steps", type=int, default=None,
                   help="timed steps of the mlp_pair / single_4096 records")
    p.add_argument("--pair-sets", type=int, default=4,
                   help="mlp_pair: step sets in flight (a stream and a plan per matrix each)")
    return p.parse_args()


def load_workloads():
    """memboost_b200/workloads.py loaded by path: importing the package would
    load its native library, which the reference arm must not."""
    spec = importlib.util.spec_from_file_location(
        "mb_workloads", os.path.join(ROOT, "memboost_b200", "workloads.py"))
    mod = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = mod  # dataclasses look their module up there
    spec.loader.exec_module(mod)
    return mod


def dist_setup():
    import torch
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if ws > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    return ws, rank, local


def barrier(ws):
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(ws, x: float) -> float:
    if ws == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


_SAMPLER = r"""
import sys, time
try:
    import pynvml
    pynvml.nvmlInit()
    try:
        h = pynvml.nvmlDeviceGetHandleByUUID(sys.argv[1])
    except Exception:
        h = pynvml.nvmlDeviceGetHandleByIndex(int(sys.argv[3]))
    mx = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
except Exception as e:
    print("error", type(e).__name__, str(e).replace(chr(10), " ")[:120], flush=True)
    sys.exit(0)
def reasons():
    for f in ("nvmlDeviceGetCurrentClocksEventReasons", "nvmlDeviceGetCurrentClocksThrottleReasons"):
        try:
            return getattr(pynvml, f)(h)
        except Exception:
            pass
    return 0
first = True
while True:
    t = time.time()
    try:
        sm = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
        try:
            pw = pynvml.nvmlDeviceGetPowerUsage(h) / 1000.0
        except Exception:
            pw = -1.0
        print(t, sm, mx, reasons(), pw, flush=True)
        if first:
            print("ready", flush=True)
            first = False
    except Exception:
        pass
    time.sleep(float(sys.argv[2]))
"""


class ClockSampler:
    """Samples this GPU's SM clock, throttle reasons and power through NVML
    every ~5 ms (read-only queries) from a separate process, started before
    the warm-up and ready once its first sample is in.  Reports the samples
    taken inside the timed window (``mark_start`` / ``mark_end``), or the
    nearest ones if the window is shorter than the period.  NVML queries slow
    the launching process down measurably at millisecond periods, hence the
    longer one."""

    PERIOD_S = 0.005

    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
               "sw_power_cap": 0x4}

    def __init__(self, device_index: int):
        self.samples = []
        self.proc = None
        self.why = ""
        self.in_window = 0
        self.lines = []
        self.t_start = self.t_end = time.time()
        try:
            import subprocess

            import torch
            uuid = "GPU-" + str(torch.cuda.get_device_properties(device_index).uuid)
            # NVML index of this device: CUDA_VISIBLE_DEVICES may renumber
            vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
            ids = [x.strip() for x in vis.split(",") if x.strip()]
            nvml_index = int(ids[device_index]) if device_index < len(ids) and \
                ids[device_index].isdigit() else device_index
            self.proc = subprocess.Popen([sys.executable, "-c", _SAMPLER, uuid,
                                          str(self.PERIOD_S), str(nvml_index)],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                                         text=True)
            # the first sample, then "ready"
            for _ in range(3):
                line = self.proc.stdout.readline().strip()
                if line == "ready":
                    break
                if not line or line.startswith("error"):
                    self.why = line or "sampler exited"
                    self.proc.kill()
                    self.proc = None
                    break
                self.lines.append(line)
        except Exception as e:
            self.why = f"{type(e).__name__}: {e}"[:120]
            self.proc = None

    def mark_start(self):
        self.t_start = time.time()

    def mark_end(self):
        self.t_end = time.time()

    def stop(self):
        if self.proc is None:
            return
        time.sleep(3 * self.PERIOD_S)  # samples after the window, for short windows
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            out, _ = self.proc.communicate()
        self.proc = None
        allsamp = []
        for line in self.lines + out.splitlines():
            try:
                t, sm, mx, rs, pw = line.split()
                allsamp.append((float(t), int(sm), int(mx), int(rs), float(pw)))
            except ValueError:
                pass
        inside = [x for x in allsamp if self.t_start <= x[0] <= self.t_end]
        self.in_window = len(inside)
        if not inside and allsamp:  # window shorter than the period: the nearest samples
            mid = 0.5 * (self.t_start + self.t_end)
            inside = sorted(allsamp, key=lambda x: abs(x[0] - mid))[:3]
        self.samples = [x[1:] for x in inside]
        if not self.samples and not self.why:
            self.why = "sampler returned no samples"

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [],
                    "unsampled_why": self.why or "no sample"}
        reasons = sorted({n for (_, _, r, _) in self.samples for n, bit in self.REASONS.items()
                          if r & bit})
        return {"sm_mhz": statistics.median(s[0] for s in self.samples),
                "sm_max_mhz": max(s[1] for s in self.samples),
                "power_w_max": round(max(s[3] for s in self.samples), 1),
                "samples": len(self.samples), "samples_in_window": self.in_window,
                "source": "NVML every ~5 ms from a separate process started before the "
                          "warm-up; samples inside the timed window (else the 3 nearest)",
                "reasons": reasons}


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        d = json.load(open(path))
        return d, "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, \
        "fallback"


def algorithmic_bytes(M: int, K: int, nnz: int, selecting: bool) -> int:
    """Compulsory HBM bytes of one quantize call: W read once (2 B/weight),
    packed 2-bit (4 B) and 4-bit (8 B) words, fp16 scale, int8 zero and uint8
    2nd-order code per (row, group) -- 3.0 B per weight -- plus hessian
    (4 B/column), 2nd-order scale+zero (3 B/chunk), CSR (6 B/outlier +
    4 B/row) and group precision (1 B/group)."""
    ng = (K + 15) // 16
    ng2 = (M * ng + 255) // 256
    return (2 * M * K + M * ng * (4 + 8 + 2 + 1 + 1) + (4 * K if selecting else 0) + 3 * ng2
            + 6 * nnz + 4 * (M + 1) + ng)


def dequant_bytes(M: int, K: int, n4: int) -> int:
    """Compulsory HBM bytes of one dequantize: the selected code words
    (4 B per 2-bit and 8 B per 4-bit (row, group)), fp16 scale and int8 zero
    per (row, group), group precision, and the fp16 output."""
    ng = (K + 15) // 16
    return M * (4 * (ng - n4) + 8 * n4) + M * ng * 3 + ng + 2 * M * K


def model_shapes(layers: int, wl):
    return [(name, M, K, wl.llama7b_model_seed(i))
            for i, (name, M, K) in enumerate(wl.llama7b_shapes(layers))]


def cpu_sample(wl, layers_shapes, device, min_rows: int = 256, frac: float = 1.0 / 16):
    """Row slices (about ``frac`` of the rows) of the first layer's seven
    matrices of the model workload, drawn on ``device`` with the model's seeds
    and copied to host memory: the CPU arms' bounded sample."""
    out = []
    for name, M, K, seed in layers_shapes[:7]:
        c = wl.llama7b_matrix(name, M, K, seed, device=device)
        r = max(min_rows, int(M * frac))
        out.append((name, c.weights[:r].cpu().numpy(), c.hessian_diag.cpu().numpy(),
                    c.ratio_4bit))
    return out


def time_oracle(oracle, sample, seconds: float):
    """Repeats the oracle over the sample for about ``seconds``; GB/s of fp16."""
    n, nbytes, t0 = 0, 0, time.perf_counter()
    while True:
        for _, w, h, r in sample:
            oracle.quantize(w, r, h, nthreads=0)
            nbytes += 2 * w.size
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds or n >= 200:
            return nbytes / el / 1e9, n, el


def cpu_baseline(wl, shapes, device, seconds=12.0):
    from oracle import oracle
    oracle.build()
    sample = cpu_sample(wl, shapes, device)
    v, n, el = time_oracle(oracle, sample, seconds)
    rows = {name: w.shape[0] for name, w, _, _ in sample}
    return {"value": round(v, 4), "unit": UNIT, "cores": os.cpu_count(), "kind": "port",
            "sample": f"oracle/mb_oracle.cpp (C++ restatement of the reference algorithm) on "
                      f"{os.cpu_count()} host threads, {n} passes over row slices of layer 0 "
                      f"({rows}), {el:.1f} s"}


# ---------------------------------------------------------------------------
# the main line: the whole model, sharded by matrix
# ---------------------------------------------------------------------------

def run_ours(args, ws, rank, local):
    import torch

    import memboost_b200 as mb
    from memboost_b200 import _C, shard
    from memboost_b200 import workloads as wl

    dev = torch.device("cuda", local)
    clk = ClockSampler(local)
    shapes = model_shapes(args.layers, wl)
    mine = shard.lpt_partition([M * K for _, M, K, _ in shapes], ws)[rank]
    if args.per_launch is None:
        # 8 matrices per launch set, but at least one set per graph branch, so
        # that a set's serial kernel chain overlaps others at 4-8 GPUs too
        args.per_launch = max(1, min(8, len(mine) // max(1, args.branches)))
    cases = [wl.llama7b_matrix(shapes[i][0], shapes[i][1], shapes[i][2], shapes[i][3],
                               device=dev) for i in mine]
    batch = _C.QuantizeBatch([c.weights for c in cases], [c.ratio_4bit for c in cases],
                             [c.hessian_diag for c in cases], dev, branches=args.branches,
                             per_launch=args.per_launch)
    del cases
    fp16_bytes = sum(2 * M * K for (M, K) in batch.shapes)
    batch.capture()

    ev = [torch.cuda.Event() for _ in range(2)]
    last = {}

    def run_steps(n):
        for k in range(n):
            batch.launch()
            ev[k % 2].record()
            if k > 0:
                ev[(k - 1) % 2].synchronize()
                last["nnz"] = batch.nnz_host.tolist()
        ev[(n - 1) % 2].synchronize()
        res = batch.finish()
        last["nnz"] = [int(r[8].numel()) for r in res]

    run_steps(max(args.warmup, 3))
    torch.cuda.synchronize()
    barrier(ws)
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    clk.mark_start()
    t0.record()
    run_steps(args.steps)
    t1.record()
    torch.cuda.synchronize()
    clk.mark_end()
    barrier(ws)
    ms_local = t0.elapsed_time(t1)
    ms = max_over_ranks(ws, ms_local)
    total_fp16 = sum(2 * M * K for _, M, K, _ in shapes)  # every rank's share together
    value = total_fp16 * args.steps / (ms / 1e3) / 1e9

    pk, peak_kind = peaks()
    hbm = float(pk["hbm_gbs"])
    nnz = last["nnz"]
    alg_local = sum(algorithmic_bytes(M, K, n, True) for (M, K), n in zip(batch.shapes, nnz))
    alg_all = alg_local
    if ws > 1:
        import torch.distributed as dist
        t = torch.tensor([float(alg_local)], dtype=torch.float64, device=dev)
        dist.all_reduce(t)
        alg_all = float(t.item())
    achieved = alg_all / (ms / args.steps / 1e3) / 1e9  # whole job
    achieved_rank = alg_local / (ms_local / args.steps / 1e3) / 1e9
    launches_per_step = batch.kernel_launches()

    # e2e: the public API per matrix, host buffers, copies in the timed region
    e2e = None
    if args.e2e_steps > 0:
        e2e = run_e2e(args, ws, dev, batch, fp16_bytes, total_fp16)
    clk.stop()

    line = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": ws,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "fp16->u8/i32",
        "data": "synthetic (seeded N(0,0.02^2) weights, lognormal(0,1.5) hessian, drawn on the "
                "GPU; no checkpoint)",
        "config": {"workload": WORKLOAD, "layers": args.layers, "matrices": len(shapes),
                   "fp16_bytes": total_fp16, "rank0_matrices": len(batch.shapes),
                   "rank0_fp16_bytes": fp16_bytes,
                   "l2": "per-step inputs 12.95 GB (1.6 GB per rank at 8) > 126 MB L2; "
                         "not flushed",
                   "parallelism": f"{ws} ranks, matrices split by size (LPT), no collective on "
                                  "the data path",
                   "schedule": {"branches": args.branches, "per_launch": args.per_launch}},
        "roofline": {"bound": "hbm", "achieved": round(achieved / ws, 1), "peak": hbm,
                     "unit": "GB/s", "frac": round(achieved / ws / hbm, 4),
                     "peak_kind": peak_kind, "of": f"{peak_kind} hbm_gbs per GPU",
                     "traffic": int(TRAFFIC_PER_STEP_MODEL * fp16_bytes / total_fp16),
                     "traffic_what": "DRAM read+write per step of this GPU's share (ncu "
                                     "capture of one whole-model step on one GPU, L2 kept "
                                     "between kernels, scaled by the share's bytes)",
                     "kernel": "the quantize calls of a step (stats, combine, tables, encode, "
                               "extract per launch set of matrices, chained with PDL): "
                               "algorithmic bytes of the whole job per GPU / device time per "
                               "step (max over ranks)",
                     "algorithmic_bytes_per_step": int(alg_all),
                     "rank0_achieved": round(achieved_rank, 1)},
        "gpu_launches": launches_per_step * args.steps,
        "gpu_launches_what": "rank 0: stats, combine, tables, encode, extract per launch set "
                             f"of up to {args.per_launch} matrices, per step",
        "nnz_rank0": int(sum(nnz)),
        "clocks": clk.summary(),
    }
    if e2e:
        line["e2e"] = e2e
    return line, shapes, wl


def run_e2e(args, ws, dev, batch, fp16_bytes, total_fp16):
    """memboost_b200.quantize() per matrix of this rank's share with host
    buffers: upload (pinned), quantize, download of every output into pinned
    buffers, all inside the timed region.  The uploads of the whole share
    are enqueued first on a copy stream (one event per matrix), so they run
    back to back while quantize() -- which waits for its matrix's kernels to
    size the CSR arrays -- and the downloads (two alternating streams)
    follow behind them."""
    import torch

    import memboost_b200 as mb
    hw = [w.cpu().pin_memory() for w in batch.weights]
    hh = [h.cpu().pin_memory() if h is not None else None for h in batch.hess]
    h2d = sum(t.numel() * t.element_size() for t in hw) + \
        sum(t.numel() * t.element_size() for t in hh if t is not None)
    wd = [torch.empty_like(w, device=dev) for w in hw]
    hd = [torch.empty_like(h, device=dev) if h is not None else None for h in hh]
    up = torch.cuda.Stream(dev)
    streams = [torch.cuda.Stream(dev) for _ in range(2)]
    ev_up = [torch.cuda.Event() for _ in hw]
    ev_used = [torch.cuda.Event() for _ in hw]
    host_out = [dict() for _ in hw]
    d2h = {"b": 0}

    def step():
        nb = 0
        with torch.cuda.stream(up):
            for i, (w, h) in enumerate(zip(hw, hh)):
                up.wait_event(ev_used[i])  # the previous step's quantize read the buffer
                wd[i].copy_(w, non_blocking=True)
                if h is not None:
                    hd[i].copy_(h, non_blocking=True)
                ev_up[i].record(up)
        for i in range(len(hw)):
            st = streams[i % 2]
            st.wait_event(ev_up[i])
            with torch.cuda.stream(st):
                qt = mb.quantize(wd[i], batch.ratios[i], hd[i])
                ev_used[i].record(st)
                for k, v in qt.state_dict().items():
                    if not (isinstance(v, torch.Tensor) and v.is_cuda):
                        continue
                    dst = host_out[i].get(k)
                    if dst is None or dst.shape != v.shape:
                        dst = torch.empty(v.shape, dtype=v.dtype).pin_memory()
                        host_out[i][k] = dst
                    dst.copy_(v, non_blocking=True)
                    nb += v.numel() * v.element_size()
        d2h["b"] = nb

    step()
    torch.cuda.synchronize()
    barrier(ws)
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for st in streams + [up]:
        st.wait_event(e0)
    for _ in range(args.e2e_steps):
        step()
    for st in streams + [up]:
        torch.cuda.current_stream(dev).wait_stream(st)
    e1.record()
    torch.cuda.synchronize()
    ems = max_over_ranks(ws, e0.elapsed_time(e1))
    return {"value": round(total_fp16 * args.e2e_steps / (ems / 1e3) / 1e9, 3), "unit": UNIT,
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h["b"],
            "per": "rank 0 (every rank moves its own share)", "steps": args.e2e_steps,
            "ms_per_step": round(ems / args.e2e_steps, 3),
            "path": "memboost_b200.quantize() per matrix (C ABI), pinned host buffers; uploads "
                    "on a copy stream ahead of the quantize calls, downloads on 2 alternating "
                    "streams"}


# ---------------------------------------------------------------------------
# one-GPU sub-records
# ---------------------------------------------------------------------------

def sub_mlp_pair(steps=1000, warmup=5, sets=4):
    """Config 2: the Llama-7B MLP pair, QuantizePlan per matrix, every plan on
    a stream of its own (two matrices x `sets` step sets), step k + sets - 1
    enqueued before step k is finished."""
    import torch

    from memboost_b200 import _C
    from memboost_b200 import workloads as wl
    dev = torch.device("cuda", torch.cuda.current_device())
    cases = wl.mlp_7b()
    W = [c.weights.to(dev) for c in cases]
    H = [c.hessian_diag.to(dev) for c in cases]
    stream_sets = [[torch.cuda.Stream(dev) for _ in W] for _ in range(sets)]
    streams = [st for ss in stream_sets for st in ss]
    plan_sets = [[_C.QuantizePlan(*w.shape, dev, stream=st) for w, st in zip(W, ss)]
                 for ss in stream_sets]
    nnz_seen = []

    def run_steps(n):
        for k in range(n):
            for p, w, h, c in zip(plan_sets[k % sets], W, H, cases):
                p.launch(w, c.ratio_4bit, h)
            if k >= sets - 1:
                nnz_seen.append([int(r[8].numel()) for r in
                                 (p.finish() for p in plan_sets[(k - sets + 1) % sets])])
        for k in range(max(0, n - sets + 1), n):
            nnz_seen.append([int(r[8].numel()) for r in (p.finish() for p in plan_sets[k % sets])])

    run_steps(warmup)
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    for st in streams:
        st.wait_event(t0)
    run_steps(steps)
    for st in streams:
        torch.cuda.current_stream(dev).wait_stream(st)
    t1.record()
    torch.cuda.synchronize()
    ms = t0.elapsed_time(t1)
    fp16 = sum(2 * w.numel() for w in W)
    alg = [algorithmic_bytes(*w.shape, n, True) for w, n in zip(W, nnz_seen[-1])]
    pk, kind = peaks()
    ach = sum(alg) / (ms / steps / 1e3) / 1e9
    return {"workload": "mlp_7b pair: 11008x4096 + 4096x11008 fp16, 0.05% Student-t(3) "
                        "outliers, lognormal(0,1.5) hessian, ratio 0.1",
            "value": round(fp16 * steps / (ms / 1e3) / 1e9, 2), "unit": UNIT, "steps": steps,
            "ms_per_step": round(ms / steps, 4),
            "roofline": {"bound": "hbm", "achieved": round(ach, 1), "peak": pk["hbm_gbs"],
                         "frac": round(ach / pk["hbm_gbs"], 4), "of": f"{kind} hbm_gbs",
                         "traffic": TRAFFIC_PER_CALL_MLP7B,
                         "algorithmic_bytes_per_call": alg},
            "gpu_launches": 5 * len(W) * steps}


def sub_single_4096(steps=200, warmup=5):
    """Config 1: 4096x4096 (0.1% x10 outliers, hessian ones, ratio 0.1):
    quantize then dequantize per step, device-resident, and dequantize
    alone with its roofline."""
    import torch

    from memboost_b200 import _C
    from memboost_b200 import workloads as wl
    dev = torch.device("cuda", torch.cuda.current_device())
    c = wl.single_4096()
    batch = _C.QuantizeBatch([c.weights], [c.ratio_4bit], [c.hessian_diag], dev, branches=1)
    batch.capture()
    M, K = batch.shapes[0]
    out = torch.empty((M, K), dtype=torch.float16, device=dev)

    o = batch.out[0]

    def step():
        # quantize (graph replay), then dequantize of its outputs on the same
        # stream; the outlier count is read once after the timed steps
        batch.launch()
        _C.dequantize(o[0], o[1], o[2], o[3], o[7], M, K, out)

    for _ in range(warmup):
        step()
    r = batch.finish()[0]
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(steps):
        step()
    t1.record()
    torch.cuda.synchronize()
    ms = t0.elapsed_time(t1) / steps
    r = batch.finish()[0]
    nnz = int(r[8].numel())
    # dequantize alone, inputs rotated over 8 copies (larger than L2 together),
    # the 8 calls recorded once in a CUDA graph so the number is device time
    copies = [[t.clone() for t in (r[0], r[1], r[2], r[3], r[7])] for _ in range(8)]
    outs = [torch.empty((M, K), dtype=torch.float16, device=dev) for _ in range(8)]
    for i in range(16):
        a = copies[i % 8]
        _C.dequantize(a[0], a[1], a[2], a[3], a[4], M, K, outs[i % 8])
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(8):
            a = copies[i]
            _C.dequantize(a[0], a[1], a[2], a[3], a[4], M, K, outs[i])
    g.replay()
    torch.cuda.synchronize()
    d0 = torch.cuda.Event(enable_timing=True)
    d1 = torch.cuda.Event(enable_timing=True)
    reps = 50
    d0.record()
    for _ in range(reps):
        g.replay()
    d1.record()
    torch.cuda.synchronize()
    dms = d0.elapsed_time(d1) / (reps * 8)
    n4 = int(r[7].sum())
    db = dequant_bytes(M, K, n4)
    pk, kind = peaks()
    qb = algorithmic_bytes(M, K, nnz, True)
    return {"workload": "single 4096x4096 fp16 N(0,0.02^2) seed 0, 0.1% x10 outliers, "
                        "hessian ones, ratio 0.1: quantize (graph replay) + dequantize",
            "value": round(2 * M * K / (ms / 1e3) / 1e9, 2), "unit": UNIT,
            "ms_per_step": round(ms, 4), "nnz": nnz, "steps": steps,
            "quantize_plus_dequantize_bytes": qb + db,
            "l2": "the same 32 MB matrix every step: largely L2-resident (no roofline claim)",
            "dequantize": {"ms": round(dms, 4),
                           "value": round(2 * M * K / (dms / 1e3) / 1e9, 1), "unit": UNIT,
                           "roofline": {"bound": "hbm", "algorithmic_bytes": db,
                                        "achieved": round(db / (dms / 1e3) / 1e9, 1),
                                        "peak": pk["hbm_gbs"],
                                        "frac": round(db / (dms / 1e3) / 1e9 / pk["hbm_gbs"], 4),
                                        "of": f"{kind} hbm_gbs",
                                        "l2": "8 rotated input/output sets (8 x 41 MB)",
                                        "timing": "CUDA-graph replay of the 8 calls"}}}


def sub_gptq(tokens=262144, reps=2, hessian_only=False):
    """Config 4: one Llama-7B layer's GPTQ (4 tcgen05 Hessians over `tokens`
    calibration tokens, 4 inverses, 7 GPTQ updates, 7 quantize calls), s per
    layer; and the Hessians alone in TFLOP/s of N*K*(K+1).  hessian_only
    skips the layer timing (a small case for profiling the Hessian kernel)."""
    import torch

    from memboost_b200 import gptq
    from memboost_b200 import workloads as wl
    dev = torch.device("cuda", torch.cuda.current_device())
    weights, inputs = wl.gptq_layer(tokens=tokens, device=dev)
    torch.cuda.synchronize()
    s_layer = None
    if not hessian_only:
        gptq.quantize_layer(weights, inputs)  # warm-up
        torch.cuda.synchronize()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record()
        for _ in range(reps):
            gptq.quantize_layer(weights, inputs)
        t1.record()
        torch.cuda.synchronize()
        s_layer = round(t0.elapsed_time(t1) / 1e3 / reps, 4)
    hres = {}
    flops_all, ms_all = 0.0, 0.0
    for key, x in inputs.items():
        K = x.shape[1]
        H = torch.empty((K, K), dtype=torch.float32, device=dev)
        gptq.hessian(x, alpha=1.0 / x.shape[0], out=H)
        torch.cuda.synchronize()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        n = 3
        a.record()
        for _ in range(n):
            gptq.hessian(x, alpha=1.0 / x.shape[0], out=H)
        b.record()
        torch.cuda.synchronize()
        ms = a.elapsed_time(b) / n
        fl = float(x.shape[0]) * K * (K + 1)
        flops_all += fl
        ms_all += ms
        hres[key] = {"K": K, "ms": round(ms, 3), "tflops": round(fl / (ms / 1e3) / 1e12, 1)}
    pk, kind = peaks()
    tf = flops_all / (ms_all / 1e3) / 1e12
    return {"workload": f"GPTQ of one Llama-7B layer: calibration X {tokens} tokens bf16 "
                        "(Student-t(4)/sqrt(4096), 1% channels x20) for K=4096 (3 inputs) and "
                        "11008 (down_proj); H=X^T X fp32; block 128; ratio 0.1",
            "s_per_layer": s_layer, "reps": reps,
            "hessian": {"per_input": hres, "tflops": round(tf, 1),
                        "flops_per_layer": flops_all, "ms_per_layer": round(ms_all, 3),
                        "roofline": {"bound": "tensor", "achieved": round(tf, 1),
                                     "peak": pk.get("bf16_tflops"), "unit": "TFLOP/s",
                                     "frac": round(tf / float(pk.get("bf16_tflops", 1590.0)), 4),
                                     "of": f"{kind} bf16_tflops (burst: kernels timed alone)",
                                     "frac_sustained": round(
                                         tf / float(pk.get("bf16_tflops_sustained", 1400.0)), 4),
                                     "sustained_note": "the K = 11008 Hessian runs ~30 ms per "
                                                       "call, long enough for the power cap",
                                     "flops": "N*K*(K+1) per Hessian (symmetric)"}}}


def sub_qgemv(reps=50, copies=8):
    """GEMV over the packed format (memboost_b200.qgemv, outliers applied) on
    the quantized MLP pair: `copies` quantized copies of each matrix rotated
    (more than the L2 together), the calls recorded once in a CUDA graph so
    the number is device time; roofline from the bytes the kernel must read."""
    import torch

    import memboost_b200 as mb
    from memboost_b200 import workloads as wl
    dev = torch.device("cuda", torch.cuda.current_device())
    pk, kind = peaks()
    out = {}
    for c in wl.mlp_7b():
        M, K = c.weights.shape
        w, h = c.weights.to(dev), c.hessian_diag.to(dev)
        qts = [mb.quantize(w, c.ratio_4bit, h) for _ in range(copies)]
        x = (torch.randn(K, generator=torch.Generator().manual_seed(1)) * 0.1).half().to(dev)
        ys = [torch.empty(M, device=dev) for _ in qts]
        ng = (K + 15) // 16
        n4 = int(qts[0].group_precision.sum())
        nnz = int(qts[0].nnz)
        # code words of each group's own precision, scale, zero, precision, x,
        # y, row pointers, CSR
        alg = M * ((ng - n4) * 4 + n4 * 8 + ng * 3) + ng + 2 * K + 4 * M + 4 * (M + 1) + 6 * nnz
        for q, y in zip(qts, ys):
            mb.qgemv(q, x, out=y)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for q, y in zip(qts, ys):
                mb.qgemv(q, x, out=y)
        g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / (reps * copies)
        out[f"{M}x{K}"] = {"us": round(us, 2), "algorithmic_bytes": alg,
                           "achieved": round(alg / us / 1e3, 1),
                           "frac": round(alg / us / 1e3 / pk["hbm_gbs"], 4),
                           "fp16_gemv_equiv_gbs": round(2 * M * K / us / 1e3, 1)}
        del qts, ys, g
    return {"what": "y = W x from the packed words (mb_qgemv), outliers written back; "
                    f"{copies} rotated copies, CUDA-graph replay", "of": f"{kind} hbm_gbs",
            **out}


def sub_rowsplit(ws, rank, steps=5, warmup=2):
    """Config 5: the Llama-70B MLP pair (28672x8192 and 8192x28672, 0.2% x10
    outliers, lognormal(0, 2) hessian, ratio 0.25) with each matrix's rows
    split over the ranks (memboost_b200.rowsplit: records all-gathered over
    NCCL, identical selection on every rank, pending groups settled from
    gathered column strips, slab encodes, CSR offsets all-gathered); at one
    GPU the plain quantize of each whole matrix.  All ranks take part; the
    step time is the max over ranks."""
    import torch

    from memboost_b200 import _C, rowsplit
    from memboost_b200 import workloads as wl
    dev = torch.device("cuda", torch.cuda.current_device())
    mats = []
    for i, (M, K) in enumerate(((28672, 8192), (8192, 28672))):
        g = torch.Generator(device=dev)
        g.manual_seed(5 + i)
        w = torch.randn((M, K), generator=g, device=dev) * 0.015
        idx = torch.randint(0, M * K, (int(round(M * K * 0.002)),), generator=g, device=dev)
        w.view(-1)[idx] *= 10.0
        h = torch.randn((K,), generator=g, device=dev).mul_(2.0).exp_()
        mats.append((w.half(), h))
        del w
    comm = rowsplit.DistComm() if ws > 1 else None
    slabs = []
    for w, h in mats:
        b = rowsplit.slab_bounds(w.shape[0], w.shape[1], ws)[rank]
        slabs.append((w[b[0]:b[1]].contiguous(), h, w.shape[0], w.shape[1]))
    info = {}

    def step():
        for j, (ws_, h, M, K) in enumerate(slabs):
            if comm is None:
                r = _C.quantize(ws_, 0.25, h)
                info[j] = (0, 0)
            else:
                r = rowsplit.quantize_rows(ws_, M, K, 0.25, h, comm)
                info[j] = (r.n_pending, r.need)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    barrier(ws)
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(steps):
        step()
    t1.record()
    torch.cuda.synchronize()
    ms = max_over_ranks(ws, t0.elapsed_time(t1)) / steps
    fp16 = sum(2 * w.numel() for w, _ in mats)
    return {"workload": "mlp_70b pair: 28672x8192 + 8192x28672 fp16 N(0,0.015^2), 0.2% x10 "
                        "outliers, lognormal(0,2) hessian, ratio 0.25; rows split over the ranks",
            "value": round(fp16 / (ms / 1e3) / 1e9, 2), "unit": UNIT, "ms_per_step": round(ms, 3),
            "n_gpus": ws, "steps": steps,
            "pending_groups": [info[j][0] for j in range(len(mats))],
            "path": "memboost_b200.rowsplit.quantize_rows (NCCL all-gathers)" if ws > 1 else
                    "memboost_b200._C.quantize on each whole matrix"}


def sub_gptq_stream(ws, rank, n_layers=2):
    """Layer-streaming GPTQ of the Llama-2-7B-shaped decoder (synthetic
    weights, 128 x 2048 calibration tokens): per layer the calibration
    forward with tcgen05 Hessians, GPTQ + quantize of the seven projections
    and the re-forward through the quantized layer; with several ranks the
    samples, Hessians, inverses and GPTQ rows are split."""
    import torch

    from memboost_b200 import llama, rowsplit
    comm = rowsplit.DistComm() if ws > 1 else None
    cfg = llama.LlamaConfig()
    _, st = llama.quantize_llama_synthetic(cfg, n_samples=128, seq_len=2048, comm=comm,
                                           n_layers=n_layers)
    sec = [max_over_ranks(ws, s) for s in st["seconds_per_layer"]]
    return {"workload": "layer-streaming GPTQ, Llama-2-7B-shaped layers (synthetic weights), "
                        "128 x 2048 calibration tokens, ratio 0.1",
            "layers": n_layers, "seconds_per_layer": [round(x, 3) for x in sec],
            "s_per_layer_after_first": round(sum(sec[1:]) / max(1, len(sec) - 1), 3),
            "compression_ratio": round(st["compression_ratio"], 3), "n_gpus": ws}


# ---------------------------------------------------------------------------
# reference arm
# ---------------------------------------------------------------------------

def run_reference_arm(args, ws, rank, local):
    """The reference algorithm on the host cores (oracle port of
    core/quantize.cu + core/torch_ops.cu), on row slices of the same model;
    as context the reference's own CUDA kernels (oracle/_ref) on layer 0 and
    its GPTQ layer loop (models/llama.py:234-294 restated in torch ops) on
    this GPU.  Nothing of memboost_b200's native library is loaded."""
    import torch

    from oracle import oracle
    wl = load_workloads()
    oracle.build()
    dev = torch.device("cuda", local)
    shapes = model_shapes(args.layers, wl)
    total_fp16 = sum(2 * M * K for _, M, K, _ in shapes)
    full = cpu_sample(wl, shapes, dev, frac=1.0)
    t_one = time.perf_counter()
    for _, w, h, r in full:
        oracle.quantize(w[:256], r, h, nthreads=0)
    t_row = (time.perf_counter() - t_one) / 256 / len(full)
    # bounded sample per step: the timed steps together take about a minute
    per_step_s = min(6.0, 60.0 / max(1, args.steps))
    rows = max(64, int(per_step_s / max(t_row, 1e-9)))
    sample = [(n, np.ascontiguousarray(w[:min(rows, w.shape[0])]), h, r) for n, w, h, r in full]
    step_bytes = sum(2 * w.size for _, w, _, _ in sample)
    for _ in range(args.warmup):
        for _, w, h, r in sample:
            oracle.quantize(w, r, h, nthreads=0)
    a = time.perf_counter()
    for _ in range(args.steps):
        for _, w, h, r in sample:
            oracle.quantize(w, r, h, nthreads=0)
    el = time.perf_counter() - a
    value = step_bytes * args.steps / el / 1e9
    rows_of = {n: w.shape[0] for n, w, _, _ in sample}
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": UNIT,
        "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(el / args.steps * 1e3, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "fp16->u8/i32",
        "data": "synthetic (seeded N(0,0.02^2) weights, lognormal(0,1.5) hessian, drawn on the "
                "GPU; no checkpoint)",
        "config": {"workload": WORKLOAD, "layers": args.layers, "matrices": len(shapes),
                   "fp16_bytes": total_fp16, "per_step_sample_rows": rows_of},
        "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": os.cpu_count(),
                         "kind": "port",
                         "sample": f"oracle/mb_oracle.cpp (the reference algorithm restated "
                                   f"in C++) on {os.cpu_count()} host threads, rows {rows_of} "
                                   f"of layer 0 of the model per step"},
        "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    # context: the reference's own CUDA kernels, built from its sources, on layer 0
    try:
        from oracle import build_ref
        ref = build_ref.load()
        cases = [wl.llama7b_matrix(n, M, K, s, device=dev) for n, M, K, s in shapes[:7]]
        for _ in range(2):
            for c in cases:
                ref.quantize(c.weights, c.ratio_4bit, c.hessian_diag)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n = 3
        e0.record()
        for _ in range(n):
            for c in cases:
                ref.quantize(c.weights, c.ratio_4bit, c.hessian_diag)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        fp16 = sum(2 * c.weights.numel() for c in cases)
        line["reference_cuda_b200"] = {
            "value": round(fp16 * n / (ms / 1e3) / 1e9, 3), "unit": UNIT,
            "ms_per_layer": round(ms / n, 3),
            "what": "reference core/*.cu compiled for sm_100a (oracle/build_ref.py), "
                    "_C.quantize on layer 0's seven matrices, CUDA events, device-resident"}
        del cases
    except Exception as e:  # not built here
        line["reference_cuda_b200"] = {"unavailable": str(e)[:200]}
    if not args.no_sub:
        try:
            line["reference_gptq_layer"] = reference_gptq_layer(wl, dev)
        except Exception as e:
            line["reference_gptq_layer"] = {"unavailable": str(e)[:200]}
    return line


def reference_gptq_layer(wl, dev, tokens=262144):
    """The reference's per-layer GPTQ on this GPU in its own torch terms: H
    accumulated as fp32 x^T x per 2048-token sample (models/llama.py:523-528),
    the damped Cholesky inverse (llama.py:177-203, torch.linalg), group
    precision by torch sum + topk (llama.py:209-231) and the column loop of
    gptq_quantize (llama.py:234-294, restated op for op in oracle/gptq_torch);
    the final memboost.quantize calls are left out (timed with our arm)."""
    import torch

    from oracle import gptq_torch
    weights, inputs = wl.gptq_layer(tokens=tokens, device=dev)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        inv = {}
        for key, x in inputs.items():
            K = x.shape[1]
            H = torch.zeros((K, K), dtype=torch.float32, device=dev)
            for s0 in range(0, x.shape[0], 2048):
                xf = x[s0:s0 + 2048].float()
                H.add_(xf.T @ xf)
            H.div_(x.shape[0])
            d = H.diagonal()
            d.add_(max((0.01 * d.abs().max()).item(), 1e-6))
            Hinv = torch.cholesky_inverse(torch.linalg.cholesky(H))
            h_diag = Hinv.diag().clone()
            Hinv.diagonal().add_(1e-8)
            inv[key] = (h_diag, torch.linalg.cholesky(Hinv, upper=True))
        t_h = time.perf_counter() - t0
        groups = {"self_attn.q_proj": "attn", "self_attn.k_proj": "attn",
                  "self_attn.v_proj": "attn", "self_attn.o_proj": "o", "mlp.gate_proj": "mlp",
                  "mlp.up_proj": "mlp", "mlp.down_proj": "down"}
        for name, W in weights.items():
            h_diag, hc = inv[groups[name]]
            M, K = W.shape
            ng = K // 16
            sens = (W.pow(2) * (1.0 / h_diag.clamp(min=1e-8)).unsqueeze(0)).view(M, ng, 16).sum(
                dim=(0, 2))
            gp = torch.zeros(ng, dtype=torch.uint8, device=dev)
            gp[sens.topk(int(0.1 * ng)).indices] = 1
            gptq_torch.gptq_quantize(W, hc, gp)
        torch.cuda.synchronize()
        total = time.perf_counter() - t0
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    return {"s_per_layer": round(total, 3), "hessians_and_inverses_s": round(t_h, 3),
            "what": "reference GPTQ steps of models/llama.py in torch on this GPU (fp32 "
                    "Hessian per 2048-token sample, cholesky inverse, column loop); "
                    "memboost.quantize calls not included"}


def main():
    args = parse()
    ws, rank, local = dist_setup()
    if args.impl == "reference":
        if rank == 0:
            print(json.dumps(run_reference_arm(args, ws, rank, local)), flush=True)
        return
    if args.only is not None:
        kw = {} if args.sub_steps is None else {"steps": args.sub_steps}
        if args.only in ("mlp_pair", "single_4096", "qgemv", "gptq_layer", "hessian") and ws > 1:
            raise SystemExit(f"--only {args.only} is a one-GPU record")
        rec = {"mlp_pair": lambda: sub_mlp_pair(sets=args.pair_sets, **kw),
               "single_4096": lambda: sub_single_4096(**kw),
               "gptq_layer": lambda: sub_gptq(tokens=args.tokens),
               "hessian": lambda: sub_gptq(tokens=args.tokens, hessian_only=True),
               "qgemv": sub_qgemv,
               "rowsplit": lambda: sub_rowsplit(ws, rank),
               "gptq_stream": lambda: sub_gptq_stream(ws, rank)}[args.only]()
        if rank == 0:
            print(json.dumps({args.only: rec}), flush=True)
        if ws > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        return
    line, shapes, wl = run_ours(args, ws, rank, local)
    if not args.no_sub:
        import torch
        torch.cuda.empty_cache()
        if ws == 1:
            line["mlp_pair"] = sub_mlp_pair()
            line["single_4096"] = sub_single_4096()
            line["gptq_layer"] = sub_gptq()
            line["qgemv"] = sub_qgemv()
        torch.cuda.empty_cache()
        line["mlp_70b_rowsplit"] = sub_rowsplit(ws, rank)
        torch.cuda.empty_cache()
        line["gptq_stream"] = sub_gptq_stream(ws, rank)
    if rank == 0:
        if ws == 1 and not args.no_cpu_baseline:
            import torch
            line["cpu_baseline"] = cpu_baseline(wl, shapes, torch.device("cuda", local))
        print(json.dumps(line), flush=True)
    if ws > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
