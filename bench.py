#!/usr/bin/env python
"""Benchmark: memboost quantize throughput on B200 (FP16 GB/s ingested).

One step = quantize the Llama-7B MLP-shaped pair (11008x4096 and 4096x11008
fp16, N(0, 0.02^2) with 0.05% Student-t(3) outliers, lognormal(0, 1.5)
hessian_diag, ratio_4bit 0.1) -- synthetic, seeded, generated on the CPU.
At N GPUs every rank quantizes its own copy (weak scaling, no collective on
the data path); rank 0 prints one JSON line.

  value      device-resident throughput: inputs already in HBM, the
             QuantizePlan path (launch both matrices, read their outlier
             counts, CSR extract); step k + 1 is enqueued before step k is
             finished, so host work overlaps the GPU
  e2e        the public memboost_b200.quantize() call per matrix with host
             buffers: pinned H2D copy of the weights and hessian, quantize,
             D2H of every output tensor, inside the timed region
  roofline   algorithmic bytes of a step's quantize calls (3.0 B per weight
             plus hessian, 2nd-order, CSR and precision bytes) / the device
             time per step, against MEASURED_PEAKS.json; traffic = DRAM bytes
             per call from the committed ncu summary
  cpu_baseline  the CPU oracle (C++ restatement of the reference algorithm)
             on all host cores, on the same matrices

--impl reference times the reference algorithm on the host cores (the
oracle port) for the same workload and, when the reference's own extension
is built in oracle/_ref, its CUDA kernels on this GPU.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "FP16 GB/s quantized (Llama-7B MLP pair 11008x4096 + 4096x11008)"
UNIT = "GB/s"


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=1000)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--e2e-steps", type=int, default=5)
    p.add_argument("--no-cpu-baseline", action="store_true")
    return p.parse_args()


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
    from memboost_b200 import shard
    return shard.max_over_ranks(x)


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
print("ready", flush=True)
def reasons():
    for f in ("nvmlDeviceGetCurrentClocksEventReasons", "nvmlDeviceGetCurrentClocksThrottleReasons"):
        try:
            return getattr(pynvml, f)(h)
        except Exception:
            pass
    return 0
while True:
    t = time.time()
    try:
        sm = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
        try:
            pw = pynvml.nvmlDeviceGetPowerUsage(h) / 1000.0
        except Exception:
            pw = -1.0
        print(t, sm, mx, reasons(), pw, flush=True)
    except Exception:
        pass
    time.sleep(float(sys.argv[2]))
"""


class ClockSampler:
    """Samples this GPU's SM clock, throttle reasons and power through NVML
    every ~5 ms (read-only queries) from a separate process, and reports the
    samples taken inside the timed window (``mark_start`` / ``mark_end``;
    the nearest one if the window is shorter than the period).  NVML queries
    slow the launching process down measurably at millisecond periods, hence
    the longer one."""

    PERIOD_S = 0.005

    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
               "sw_power_cap": 0x4}

    def __init__(self, device_index: int):
        self.samples = []
        self.proc = None
        self.why = ""
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
            first = self.proc.stdout.readline().strip()
            if first != "ready":
                self.why = first or "sampler exited"
                self.proc.kill()
                self.proc = None
        except Exception as e:
            self.why = f"{type(e).__name__}: {e}"[:120]
            self.proc = None

    def __enter__(self):
        self.t_start = self.t_end = time.time()
        return self

    def mark_start(self):
        self.t_start = time.time()

    def mark_end(self):
        self.t_end = time.time()

    def __exit__(self, *exc):
        if self.proc is None:
            return
        time.sleep(2 * self.PERIOD_S)  # a sample after the window, for short windows
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            out, _ = self.proc.communicate()
        allsamp = []
        for line in out.splitlines():
            try:
                t, sm, mx, rs, pw = line.split()
                allsamp.append((float(t), int(sm), int(mx), int(rs), float(pw)))
            except ValueError:
                pass
        inside = [x for x in allsamp if self.t_start <= x[0] <= self.t_end]
        self.in_window = len(inside)
        if not inside and allsamp:  # window shorter than the period: the nearest sample
            mid = 0.5 * (self.t_start + self.t_end)
            inside = [min(allsamp, key=lambda x: abs(x[0] - mid))]
        self.samples = [x[1:] for x in inside]

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"],
                    "why": self.why or "no sample"}
        reasons = sorted({n for (_, _, r, _) in self.samples for n, bit in self.REASONS.items()
                          if r & bit})
        return {"sm_mhz": statistics.median(s[0] for s in self.samples),
                "sm_max_mhz": max(s[1] for s in self.samples),
                "power_w_max": round(max(s[3] for s in self.samples), 1),
                "samples": len(self.samples), "samples_in_window": self.in_window,
                "source": "NVML every ~5 ms from a separate process, samples inside the "
                          "timed window (else the nearest)",
                "reasons": reasons}


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        d = json.load(open(path))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def profiled_traffic():
    """DRAM bytes (read + write) of one quantize call of the benchmark pair,
    from the committed ncu summary (a number, not a measurement of this run)."""
    path = os.path.join(ROOT, "profiles", "quantize_mlp7b_launches.md")
    try:
        for line in open(path):
            if line.startswith("traffic_bytes_per_call:"):
                return int(line.split(":", 1)[1])
    except OSError:
        pass
    return None


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


def cpu_baseline(cases, min_seconds=10.0):
    from oracle import oracle
    oracle.build()
    n, t0 = 0, time.perf_counter()
    nbytes = 0
    while True:
        for c in cases:
            oracle.quantize(c.weights.numpy(), c.ratio_4bit, c.hessian_diag.numpy(), nthreads=0)
            nbytes += 2 * c.weights.numel()
        n += 1
        el = time.perf_counter() - t0
        if el >= min_seconds or n >= 50:
            break
    return {"value": round(nbytes / el / 1e9, 4), "unit": UNIT, "cores": os.cpu_count(),
            "kind": "port",
            "sample": f"oracle/mb_oracle.cpp on {os.cpu_count()} host threads, {n} x the "
                      f"full pair ({'+'.join(c.name for c in cases)}), {el:.1f} s"}


def run_ours(args, ws, rank, local):
    import torch

    import memboost_b200 as mb
    from memboost_b200 import _C, workloads

    dev = torch.device("cuda", local)
    cases = workloads.mlp_7b()
    W = [c.weights.to(dev) for c in cases]
    H = [c.hessian_diag.to(dev) for c in cases]
    # two sets of plans: step k + 1 is enqueued before step k is finished
    # (its outlier count read and CSR extracted), so the GPU does not idle
    # while the host works; every step's outputs are complete inside the
    # timed region.  Every plan has a stream of its own (two matrices x two
    # sets): the matrices are independent, so one call's latency-bound
    # selection tail overlaps other calls' streaming kernels, including the
    # next step's, which would otherwise queue behind it on a shared stream.
    stream_sets = [[torch.cuda.Stream(dev) for _ in W] for _ in range(2)]
    streams = [st for ss in stream_sets for st in ss]
    plan_sets = [[_C.QuantizePlan(*w.shape, dev, stream=st) for w, st in zip(W, ss)]
                 for ss in stream_sets]
    fp16_bytes = sum(2 * w.numel() for w in W)
    nnz_seen = []

    def launch_step(k, ev=None):
        for i, (p, w, h, c) in enumerate(zip(plan_sets[k % 2], W, H, cases)):
            if ev is not None:
                p.record_on(ev[i][0])
            p.launch(w, c.ratio_4bit, h)
            if ev is not None:
                p.record_on(ev[i][1])

    def finish_step(k):
        res = [p.finish() for p in plan_sets[k % 2]]
        nnz_seen.append([int(r[8].numel()) for r in res])

    def run_steps(n, events=None):
        for k in range(n):
            launch_step(k, None if events is None else events[k])
            if k > 0:
                finish_step(k - 1)
        finish_step(n - 1)

    run_steps(max(args.warmup, 3))
    torch.cuda.synchronize()
    per_call = [[] for _ in W]
    events = [[[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in W]
              for _ in range(min(args.steps, 5))]
    barrier(ws)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        clk.mark_start()
        t0.record()
        for st in streams:  # the plans' streams start after t0 ...
            st.wait_event(t0)
        run_steps(args.steps)
        for st in streams:  # ... and t1 follows all of their work
            torch.cuda.current_stream(dev).wait_stream(st)
        t1.record()
        torch.cuda.synchronize()
        clk.mark_end()
    barrier(ws)
    ms_local = t0.elapsed_time(t1)
    ms = max_over_ranks(ws, ms_local)
    # per-call durations (informational), in an untimed pass of their own:
    # the events between launches cost host time
    n_ev = min(args.steps, 5)
    run_steps(n_ev, events)
    torch.cuda.synchronize()
    for k in range(n_ev):
        for i in range(len(W)):
            per_call[i].append(events[k][i][0].elapsed_time(events[k][i][1]))
    value = fp16_bytes * args.steps * ws / (ms / 1e3) / 1e9

    # roofline of the quantize path: the algorithmic bytes of a step's calls
    # over the device time per step (the two calls overlap on their streams;
    # call_ms, each call from its first to its last kernel, is informational)
    peak, peak_kind = peaks()
    nnz = nnz_seen[-1]
    alg = [algorithmic_bytes(*w.shape, n, True) for w, n in zip(W, nnz)]
    dur = [statistics.mean(x) for x in per_call]
    achieved = sum(alg) / (ms / args.steps / 1e3) / 1e9
    # stats (+selection), exact (tables), encode per matrix; extract when the
    # matrix has outliers
    launches_per_step = sum(3 + (1 if n > 0 else 0) for n in nnz)

    # e2e: public API, host buffers, copies in the timed region.  Each matrix
    # has a stream of its own: its upload, quantize() (which reads the
    # outlier count, waiting for that stream only) and the download of every
    # output into pinned host buffers; one matrix's download overlaps the
    # other's upload (the link is full duplex).  The step's outputs are all
    # on the host when the step's final synchronisation returns.
    e2e = None
    if args.e2e_steps > 0:
        hw = [c.weights.pin_memory() for c in cases]
        hh = [c.hessian_diag.pin_memory() for c in cases]
        h2d = sum(t.numel() * t.element_size() for t in hw + hh)
        e_streams = [torch.cuda.Stream(dev) for _ in cases]
        host_out = [dict() for _ in cases]  # pinned destinations, by state_dict key
        d2h_holder = {}

        def e2e_step(sync=True):
            # both uploads first: the link stays busy while quantize() waits
            # for a matrix's outlier count
            dev_in = []
            for wh, hhh, st in zip(hw, hh, e_streams):
                with torch.cuda.stream(st):
                    dev_in.append((wh.to(dev, non_blocking=True),
                                   hhh.to(dev, non_blocking=True)))
            for i, ((wd, hd), c, st) in enumerate(zip(dev_in, cases, e_streams)):
                with torch.cuda.stream(st):
                    qt = mb.quantize(wd, c.ratio_4bit, hd)
                    for k, v in qt.state_dict().items():
                        if not (isinstance(v, torch.Tensor) and v.is_cuda):
                            continue
                        dst = host_out[i].get(k)
                        if dst is None or dst.shape != v.shape:
                            dst = torch.empty(v.shape, dtype=v.dtype).pin_memory()
                            host_out[i][k] = dst
                        dst.copy_(v, non_blocking=True)
                    wd.record_stream(st)
            if sync:
                torch.cuda.synchronize()
            d2h_holder["bytes"] = sum(v.numel() * v.element_size() for d in host_out
                                      for v in d.values())

        for _ in range(2):
            e2e_step()
        barrier(ws)
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for st in e_streams:
            st.wait_event(e0)
        for k in range(args.e2e_steps):
            # step k's downloads overlap step k+1's uploads; the final
            # synchronisation completes every step
            e2e_step(sync=k == args.e2e_steps - 1)
        for st in e_streams:
            torch.cuda.current_stream(dev).wait_stream(st)
        e1.record()
        torch.cuda.synchronize()
        ems = max_over_ranks(ws, e0.elapsed_time(e1))
        e2e = {"value": round(fp16_bytes * args.e2e_steps * ws / (ems / 1e3) / 1e9, 3),
               "unit": UNIT, "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": d2h_holder["bytes"], "steps": args.e2e_steps,
               "ms_per_step": round(ems / args.e2e_steps, 3),
               "path": "memboost_b200.quantize() per matrix (C ABI), pinned host buffers, "
                       "one stream per matrix"}

    line = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": ws,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp16->u8/i32",
        "data": "synthetic (seeded N(0,0.02^2) + Student-t(3) outliers, lognormal hessian)",
        "config": {"workload": "mlp_7b pair: 11008x4096 + 4096x11008 fp16, ratio_4bit 0.1, "
                               "hessian_diag lognormal(0,1.5), 16-col groups",
                   "per_rank_fp16_bytes": fp16_bytes,
                   "l2": "per-step inputs 180 MB > 126 MB L2; not flushed",
                   "parallelism": f"{ws} independent ranks (weak scaling)"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                     "unit": "GB/s", "frac": round(achieved / peak, 4),
                     "peak_kind": peak_kind, "traffic": profiled_traffic(),
                     "traffic_source": "profiles/quantize_mlp7b_launches.md (ncu, one "
                                       "pipelined step, DRAM read+write per call)",
                     "kernel": "quantize calls of a step: stats (+group parameters and "
                               "selection), exact/tables, encode (+row pointers) -- 3 kernels "
                               "chained with PDL per matrix, every plan on a stream of its own "
                               "(2 matrices x 2 step sets); "
                               "device time per step",
                     "algorithmic_bytes_per_call": alg,
                     "call_ms": [round(d, 4) for d in dur]},
        "gpu_launches": launches_per_step * args.steps,
        "nnz": nnz,
        "clocks": clk.summary(),
    }
    if e2e:
        line["e2e"] = e2e
    return line, cases


def run_reference_arm(args, ws, rank, local):
    """Reference algorithm on the host cores (oracle port) + the reference's
    own CUDA kernels on this GPU when built in oracle/_ref."""
    import torch

    from memboost_b200 import workloads
    from oracle import oracle

    oracle.build()
    cases = workloads.mlp_7b()
    fp16 = sum(2 * c.weights.numel() for c in cases)
    wn = [c.weights.numpy() for c in cases]
    hn = [c.hessian_diag.numpy() for c in cases]
    t_one = time.perf_counter()
    for w, h, c in zip(wn, hn, cases):
        oracle.quantize(w, c.ratio_4bit, h, nthreads=0)
    t_one = time.perf_counter() - t_one
    # bounded sample per step: whole pair if a step is short, else row slices;
    # the timed steps together take about a minute (6 s a step at most), the
    # warm-up steps likewise
    per_step_s = min(6.0, 60.0 / max(1, args.steps))
    frac = min(1.0, per_step_s / max(t_one, 1e-6))
    rows = [max(256, int(w.shape[0] * frac)) for w in wn]
    sample = [np.ascontiguousarray(w[:r]) for w, r in zip(wn, rows)] if frac < 1 else wn
    step_bytes = sum(2 * s.size for s in sample)
    for _ in range(args.warmup):
        for s, h, c in zip(sample, hn, cases):
            oracle.quantize(s, c.ratio_4bit, h, nthreads=0)
    a = time.perf_counter()
    for _ in range(args.steps):
        for s, h, c in zip(sample, hn, cases):
            oracle.quantize(s, c.ratio_4bit, h, nthreads=0)
    el = time.perf_counter() - a
    value = step_bytes * args.steps / el / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": UNIT,
        "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(el / args.steps * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp16->u8/i32", "data": "synthetic",
        "config": {"workload": "mlp_7b pair: 11008x4096 + 4096x11008 fp16, ratio_4bit 0.1",
                   "per_step_sample_rows": rows},
        "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": os.cpu_count(),
                         "kind": "port",
                         "sample": f"oracle/mb_oracle.cpp (reference algorithm) on "
                                   f"{os.cpu_count()} host threads, rows {rows} of the pair"},
        "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    # the reference's own CUDA kernels, built from its sources, on this GPU
    try:
        from oracle import build_ref
        ref = build_ref.load()
        dev = torch.device("cuda", local)
        W = [c.weights.to(dev) for c in cases]
        H = [c.hessian_diag.to(dev) for c in cases]
        for _ in range(3):
            for w, h, c in zip(W, H, cases):
                ref.quantize(w, c.ratio_4bit, h)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n = max(3, min(args.steps, 10))
        e0.record()
        for _ in range(n):
            for w, h, c in zip(W, H, cases):
                ref.quantize(w, c.ratio_4bit, h)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        line["reference_cuda_b200"] = {
            "value": round(fp16 * n / (ms / 1e3) / 1e9, 3), "unit": UNIT,
            "ms_per_step": round(ms / n, 3),
            "what": "reference core/*.cu compiled for sm_100a (oracle/build_ref.py), "
                    "_C.quantize on the same pair, CUDA events, device-resident inputs"}
    except Exception as e:  # not built here
        line["reference_cuda_b200"] = {"unavailable": str(e)[:200]}
    return line


def main():
    args = parse()
    ws, rank, local = dist_setup()
    if args.impl == "reference":
        if rank == 0:
            print(json.dumps(run_reference_arm(args, ws, rank, local)), flush=True)
        return
    line, cases = run_ours(args, ws, rank, local)
    if rank == 0:
        if ws == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(cases)
        print(json.dumps(line), flush=True)
    if ws > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
