#!/usr/bin/env python3
"""Benchmark: effective TFLOP/s (nonzero blocks only) of BSR SpMM / SDDMM.

Default workload (N=1): BASELINE config 2, the SpMM density sweep.  A is
4096x4096 bf16 BSR with 32x32 blocks at p in {0.01, 0.05, 0.10, 0.25, 0.50},
B is 4096x4096 bf16, values uniform[-1,1] (seeded synthetic data), fp32
accumulate, bf16 C.  One step = one SpMM per density (five launches), each
preceded by an L2 flush (a 256 MiB write) so every launch reads HBM cold.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--strategy dda]
                  [--impl bsp|reference] [--workload sweep|cfg1|cfg3|cfg4|cfg5]

N > 1 (torchrun, one rank per GPU): every rank runs its own independent copy
of the sweep (its own seed); no collective touches the data path; value =
all ranks' effective FLOPs / max-over-ranks device time ("weak" scaling).
The cfg5 workload is the strong-scaling one: A's block-rows are sharded by
nonzero-block count and C row-panels are all-gathered with NCCL.

--impl reference times the reference's own CPU golden (bsr_matrix::
spmm_bfloat16, compiled from the reference sources into oracle/_ref; the
oracle restatement if that library is absent) with all host threads, on a
bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "tenstorrent-wh-blockspmm_b200")
for _p in (ROOT, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "effective TFLOP/s (nnz blocks only), BSR SpMM density sweep"
DENSITIES = [0.01, 0.05, 0.10, 0.25, 0.50]
L2_FLUSH_BYTES = 256 << 20
REF_TOTAL_BUDGET_S = 150.0
WORKLOAD_SWEEP = ("BASELINE config 2: BSR SpMM 4096x4096x4096, 32x32 blocks, "
                  "p in {0.01,0.05,0.10,0.25,0.50}")


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained"), "src": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "src": "fallback"}


# ------------------------------------------------------------- workloads --
def gen_spmm_case(M, K, N, R, C, p, seed):
    rng = np.random.default_rng(seed)
    occ = rng.random((M // R, K // C)) < p
    rp = np.concatenate([[0], np.cumsum(occ.sum(1))]).astype(np.int32)
    ci = np.nonzero(occ)[1].astype(np.int32)
    vals = f32_to_bf16(rng.uniform(-1, 1, ci.size * R * C).astype(np.float32))
    B = f32_to_bf16(rng.uniform(-1, 1, (K, N)).astype(np.float32))
    return dict(kind="spmm", M=M, K=K, N=N, R=R, C=C, p=p, rp=rp, ci=ci, vals=vals, B=B)


def spmm_flops(c):
    return 2.0 * int(c["rp"][-1]) * c["R"] * c["C"] * c["N"]


def spmm_bytes(c, esz=2):
    """Algorithmic bytes: A values + indices + each distinct B K-slice once + all of C."""
    nnzb = int(c["rp"][-1])
    ncols = np.unique(c["ci"]).size
    return (2 * nnzb * c["R"] * c["C"] + 4 * (nnzb + c["M"] // c["R"] + 1)
            + 2 * ncols * c["C"] * c["N"] + esz * c["M"] * c["N"])


def sweep_cases(rank):
    return [gen_spmm_case(4096, 4096, 4096, 32, 32, p, 1234 + 1 + 100 * rank + i)
            for i, p in enumerate(DENSITIES)]


# ---------------------------------------------------------------- clocks --
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.proc = None
        self.path = None
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(gpu_index)], stdout=self.fh, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.fh.close()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    rows.append(dict(sm=float(parts[1]), smax=float(parts[2]), power=float(parts[3]),
                                     hw=parts[5], hwt=parts[6], swt=parts[7], swp=parts[8]))
                except ValueError:
                    continue
        os.unlink(self.path)
        if not rows:
            return None
        reasons = set()
        for r in rows:
            for k, name in (("hw", "hw_slowdown"), ("hwt", "hw_thermal_slowdown"),
                            ("swt", "sw_thermal_slowdown"), ("swp", "sw_power_cap")):
                if r[k].lower().startswith("active"):
                    reasons.add(name)
        loaded = [r["sm"] for r in rows if r["power"] > 250] or [r["sm"] for r in rows]
        return {"sm_mhz": float(np.median(loaded)), "sm_max_mhz": rows[0]["smax"],
                "reasons": sorted(reasons), "samples": len(rows)}


# ------------------------------------------------------------- dist utils --
def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def init_dist(ws, local):
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    torch.cuda.set_device(local)
    if ws > 1:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return dist if ws > 1 else None


def max_over_ranks(x: float, dist) -> float:
    if dist is None:
        return x
    import torch

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(x: float, dist) -> float:
    if dist is None:
        return x
    import torch

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def barrier(dist):
    import torch

    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()


# ------------------------------------------------------------ CPU baseline --
def cpu_calibrate(cases, budget_s=12.0, threads=None):
    """Pick, per case, how many leading block-rows the CPU golden can finish
    in about budget_s / len(cases) seconds.  Returns (rows per case, kind)."""
    import oracle

    threads = threads or os.cpu_count() or 1
    kind = "reference" if oracle.ref_available() else "port"
    per_case = budget_s / len(cases)
    rows_out = []
    for c in cases:
        nbr = c["M"] // c["R"]
        rows = min(max(threads, 1), nbr)
        for _ in range(8):
            t = _cpu_time(c, rows, threads, kind)
            if t >= per_case / 2 or rows >= nbr:
                break
            rows = min(nbr, int(rows * min(16.0, max(1.5, per_case / max(t, 1e-4)))))
        rows_out.append(rows)
    return rows_out, kind


def cpu_sample_time(cases, rows, kind, threads=None):
    """Time the calibrated block-row sample of every case once.
    Returns (effective flops done, seconds, sample description)."""
    threads = threads or os.cpu_count() or 1
    total_f = total_t = 0.0
    samples = []
    for c, r in zip(cases, rows):
        total_t += _cpu_time(c, r, threads, kind)
        total_f += 2.0 * int(c["rp"][r]) * c["R"] * c["C"] * c["N"]
        samples.append(f"p={c['p']}: {r}/{c['M'] // c['R']} block-rows")
    return total_f, total_t, "; ".join(samples)


def cpu_reference_time(cases, budget_s=12.0, threads=None):
    """Time the reference golden (oracle/_ref) or, if absent, the oracle
    restatement, on a bounded block-row sample of each case.  Returns
    (flops_done, seconds, kind, cores, sample_description)."""
    threads = threads or os.cpu_count() or 1
    rows, kind = cpu_calibrate(cases, budget_s, threads)
    f, t, sample = cpu_sample_time(cases, rows, kind, threads)
    return f, t, kind, threads, sample


def _cpu_time(c, rows, threads, kind):
    import oracle

    if kind == "reference":
        return oracle.ref_spmm_timed(c["rp"], c["ci"], c["vals"], c["M"], c["K"], c["R"], c["C"],
                                     c["B"], c["N"], (0, rows), threads)
    t0 = time.perf_counter()
    oracle.spmm_bf16(c["rp"], c["ci"], c["vals"], c["M"], c["K"], c["R"], c["C"], c["B"], c["N"],
                     threads=threads, rows=(0, rows))
    return time.perf_counter() - t0


# --------------------------------------------------------------- our arm --
def run_bsp(args):
    import torch

    import bsp

    ws, rank, local = dist_env()
    dist = init_dist(ws, local)
    peaks = load_peaks()
    dev = bsp.device(local)
    strategy = bsp.STRATEGIES[args.strategy]
    cases = sweep_cases(rank)
    stream = torch.cuda.current_stream()
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device="cuda")

    runs = []
    for c in cases:
        A = bsp.DeviceBSR.from_host(c["M"], c["K"], c["R"], c["C"], c["rp"], c["ci"], c["vals"], local)
        B = bsp.to_device_bf16(c["B"], local)
        Cout = torch.empty((c["M"], c["N"]), dtype=torch.bfloat16, device="cuda")
        plan = bsp.SpmmPlan(dev, A, c["N"], strategy)
        runs.append(dict(case=c, A=A, B=B, C=Cout, plan=plan, flops=spmm_flops(c),
                         bytes=spmm_bytes(c), times=[]))

    def step(record):
        for r in runs:
            flush.zero_()
            if record:
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                e0.record(stream)
            r["plan"].execute(r["A"], r["B"], r["C"], stream)
            if record:
                e1.record(stream)
                r["times"].append((e0, e1))

    for _ in range(args.warmup):
        step(False)
    dev.synchronize()
    # quick self-check of the first density against the oracle on a few rows
    barrier(dist)
    sampler = ClockSampler(local) if rank == 0 else None
    for _ in range(args.steps):
        step(True)
    barrier(dist)
    clocks = sampler.stop() if sampler else None
    dev.synchronize()

    per = []
    total_t = 0.0
    total_f = 0.0
    for r in runs:
        ts = [a.elapsed_time(b) * 1e-3 for a, b in r["times"]]
        t = float(np.mean(ts))
        total_t += sum(ts)
        total_f += r["flops"] * len(ts)
        c = r["case"]
        t_tc = r["flops"] / (peaks["bf16_tflops"] * 1e12)
        t_hbm = r["bytes"] / (peaks["hbm_gbs"] * 1e9)
        per.append(dict(p=c["p"], nnzb=int(c["rp"][-1]), ms=t * 1e3,
                        tflops=r["flops"] / t / 1e12, gbs=r["bytes"] / t / 1e9,
                        bound="tensor" if t_tc >= t_hbm else "hbm",
                        roofline_frac=max(t_tc, t_hbm) / t, plan=r["plan"].info()))
    t_all = max_over_ranks(total_t, dist)
    f_all = sum_over_ranks(total_f, dist)
    value = f_all / t_all / 1e12

    # dominant kernel = the launch with the largest share of device time
    dom = max(per, key=lambda d: d["ms"])
    dom_run = runs[[d["p"] for d in per].index(dom["p"])]
    if dom["bound"] == "tensor":
        roof = {"bound": "tensor", "achieved": dom["tflops"], "peak": peaks["bf16_tflops"],
                "unit": "TFLOP/s", "frac": dom["tflops"] / peaks["bf16_tflops"]}
    else:
        roof = {"bound": "hbm", "achieved": dom["gbs"], "peak": peaks["hbm_gbs"],
                "unit": "GB/s", "frac": dom["gbs"] / peaks["hbm_gbs"]}
    roof["traffic"] = traffic_for(dom["p"], dom_run["bytes"])
    roof["peak_src"] = peaks["src"]
    variant = dom["plan"].get("variant", 0)
    roof["kernel"] = f"{'spmm_rowstack_tcgen05' if variant == 1 else 'spmm_bsr_tcgen05'} p={dom['p']}"
    roof["algorithmic"] = dom_run["bytes"] if dom["bound"] == "hbm" else dom_run["flops"]

    # ---- e2e through the host-buffer C ABI (pinned host memory) ----
    e2e = run_e2e(args, runs, dev, strategy, dist)

    # ---- CPU baseline (rank 0, N=1 only) ----
    cpu = None
    if ws == 1 and not args.no_cpu:
        f, t, kind, cores, sample = cpu_reference_time(cases, budget_s=args.cpu_budget)
        cpu = {"value": f / t / 1e12, "unit": "TFLOP/s", "cores": cores, "kind": kind,
               "sample": sample + " of each density; golden bsr_matrix::spmm_bfloat16"}

    out = {
        "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": ws, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": t_all / args.steps * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded numpy: Bernoulli block occupancy, uniform[-1,1] values)",
        "config": {"workload": WORKLOAD_SWEEP, "strategy": args.strategy,
                   "c_dtype": "bf16", "accumulate": "fp32",
                   "l2": "flushed (256 MiB write) before every timed launch",
                   "per_rank": "independent copy of the sweep per rank" if ws > 1 else None},
        "roofline": roof, "cpu_baseline": cpu, "e2e": e2e,
        "gpu_launches": args.steps * len(runs), "clocks": clocks,
        "sweep": [{k: v for k, v in d.items() if k != "plan"} | {"units": d["plan"]["units"]}
                  for d in per],
    }
    if rank == 0:
        print(json.dumps(out), flush=True)
    for r in runs:
        r["plan"].close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def run_e2e(args, runs, dev, strategy, dist):
    """Same metric end to end: pinned host inputs -> H2D -> plan -> SpMM -> D2H."""
    import torch

    import bsp

    host = []
    h2d = d2h = 0
    for r in runs:
        c = r["case"]

        def pin(a):
            t = torch.from_numpy(np.ascontiguousarray(a)).pin_memory()
            return t.numpy()

        hc = dict(rp=pin(c["rp"]), ci=pin(c["ci"]), vals=pin(c["vals"]), B=pin(c["B"]),
                  out=torch.empty((c["M"], c["N"]), dtype=torch.int16).pin_memory().numpy().view(np.uint16))
        host.append((c, hc))
        h2d += hc["rp"].nbytes + hc["ci"].nbytes + hc["vals"].nbytes + hc["B"].nbytes
        d2h += hc["out"].nbytes
    e2e_steps = max(1, min(args.steps, args.e2e_steps))

    def one():
        for c, hc in host:
            bsp.spmm_host(c["M"], c["K"], c["R"], c["C"], hc["rp"], hc["ci"], hc["vals"], hc["B"],
                          c["N"], strategy=strategy, dev=dev, out=hc["out"])

    one()  # warm (workspace growth)
    barrier(dist)
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        one()
    t = time.perf_counter() - t0
    t = max_over_ranks(t, dist)
    f = sum_over_ranks(sum(r["flops"] for r in runs) * e2e_steps, dist)
    return {"value": f / t / 1e12, "unit": "TFLOP/s", "h2d_bytes_per_step": int(h2d),
            "d2h_bytes_per_step": int(d2h), "steps": e2e_steps,
            "path": "bsp_spmm_host (C ABI, host buffers, synchronous)"}


def traffic_for(p, algorithmic_bytes):
    """DRAM bytes per launch of the dominant kernel from the committed ncu
    summary (profiles/spmm_traffic.json), if one was captured for this p."""
    path = os.path.join(ROOT, "profiles", "spmm_traffic.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return d.get(str(p))
    except Exception:
        return None


# --------------------------------------------------------- reference arm --
def run_reference(args):
    """The reference arm: the reference's CPU golden on this box's host cores.
    The whole run (calibration, warm-up and timed steps) is held to about
    REF_TOTAL_BUDGET_S seconds by shrinking each step's block-row sample."""
    ws, rank, local = dist_env()
    if rank != 0:
        return
    cases = sweep_cases(0)
    threads = os.cpu_count() or 1
    per_step = max(0.25, min(args.cpu_budget, REF_TOTAL_BUDGET_S / (args.steps + args.warmup + 2)))
    rows, kind = cpu_calibrate(cases, budget_s=per_step, threads=threads)
    sample = ""
    for _ in range(args.warmup):
        cpu_sample_time(cases, rows, kind, threads)
    tot_f = tot_t = 0.0
    for _ in range(args.steps):
        f, t, sample = cpu_sample_time(cases, rows, kind, threads)
        tot_f += f
        tot_t += t
    v = tot_f / tot_t / 1e12
    out = {"impl": "reference", "metric": METRIC, "value": v, "unit": "TFLOP/s", "n_gpus": ws,
           "steps": args.steps, "warmup": args.warmup,
           "ms_per_step": tot_t / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
           "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
           "config": {"workload": WORKLOAD_SWEEP, "strategy": "cpu golden"},
           "cpu_baseline": {"value": v, "unit": "TFLOP/s", "cores": threads, "kind": kind,
                            "sample": sample + " of each density, every step"},
           "e2e": {"value": v, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="bsp", choices=["bsp", "reference"])
    ap.add_argument("--strategy", default="dda", choices=["naive", "snf", "dda"])
    ap.add_argument("--cpu-budget", type=float, default=12.0)
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--no-cpu", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_bsp(args)


if __name__ == "__main__":
    main()
