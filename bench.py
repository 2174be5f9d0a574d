#!/usr/bin/env python3
"""Benchmark: effective TFLOP/s (nonzero blocks only) of BSR SpMM / SDDMM.

Workloads (seeded synthetic data of the stated shapes and
value distributions, generated with numpy):

  sweep (default)  config 2: A 4096x4096 bf16 BSR, 32x32 blocks, independent
                   block occupancy p in {0.01, 0.05, 0.10, 0.25, 0.50}, B dense
                   4096x4096, uniform[-1,1]; one step = one SpMM per density.
  cfg1             config 1: A 1024x1024, p=0.10, B 1024x256.
  cfg3             config 3: SDDMM, A 4096x256 and B 256x4096 N(0,1)/16, mask
                   4096x4096 with 32x32 blocks at p=0.05 (pattern only).
  cfg4             config 4: attention-shaped pair at sequence 16384, head 128,
                   32x32 blocks: mask = band of 8 blocks + 4 global block-columns
                   + Zipf(1.2) random blocks per block-row (capped at 64);
                   one step = SDDMM (Q K^T under the mask) + SpMM (P V), P having
                   the mask's pattern and row-normalised uniform[0,1] values.
  cfg5             config 5: A 65536x65536, 64x64 blocks, Zipf(1.1) block-row
                   counts at 1% mean density, B 65536x8192 uniform[-1,1]; A's
                   block-rows are sharded over the GPUs by nonzero-block count
                   and the C row-panels exchanged over NCCL (strong scaling).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--workload sweep]
                  [--strategy auto] [--impl bsp|reference]

fp32 accumulate, bf16 outputs.  Every timed launch is preceded by an L2 flush
(a 256 MiB write) and timed with CUDA events on the launching stream.  For
N > 1 (torchrun, one rank per GPU) the sweep/cfg1/cfg3/cfg4 workloads run an
independent copy per rank (own seed, no collective on the data path: "weak"
scaling); cfg5 splits one problem ("strong" scaling).  value = all ranks'
effective FLOPs / max-over-ranks device time.

--impl reference times the reference's own CPU golden (bsr_matrix::
spmm_bfloat16 / sddmm compiled from the reference sources into oracle/_ref;
the oracle restatement when that library is absent) on all host threads, on
a bounded block-row sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "tenstorrent-wh-blockspmm_b200")
for _p in (ROOT, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "effective TFLOP/s (nnz blocks only), BSR SpMM density sweep"
METRICS = {
    "sweep": METRIC,
    "cfg1": "effective TFLOP/s (nnz blocks only), BSR SpMM",
    "cfg3": "effective TFLOP/s (nnz blocks only), BSR SDDMM",
    "cfg4": "effective TFLOP/s (nnz blocks only), BSR SDDMM + SpMM attention pair",
    "cfg5": "effective TFLOP/s (nnz blocks only), multi-GPU BSR SpMM with C all-gather",
    "attn": "effective TFLOP/s (nnz blocks only), fused SDDMM -> row softmax -> SpMM attention step",
    "spgemm": "effective TFLOP/s (stored block products only), BSR x BSR -> BSR SpGEMM",
    "spgemm_rand": "effective TFLOP/s (stored block products only), BSR x BSR -> BSR SpGEMM",
}
WORKLOAD_DESC = {
    "sweep": "BASELINE config 2: BSR SpMM 4096x4096x4096, 32x32 blocks, p in {0.01,0.05,0.10,0.25,0.50}",
    "cfg1": "BASELINE config 1: BSR SpMM 1024x1024 (p=0.10, 32x32 blocks) x 1024x256",
    "cfg3": "BASELINE config 3: BSR SDDMM 4096x256 x 256x4096 under a 4096x4096 mask, 32x32 blocks, p=0.05",
    "cfg4": "BASELINE config 4: SDDMM Q K^T + SpMM P V, seq 16384, head 128, 32x32 blocks, band+global+Zipf mask",
    "cfg5": "BASELINE config 5: BSR SpMM 65536x65536 (64x64 blocks, Zipf(1.1) rows, 1% mean) x 65536x8192, "
            "row panels sharded by nnz blocks (C row-sharded in value; replicated on every GPU by the "
            "kernel's epilogue peer stores under 'replicated')",
    "attn": "BASELINE config 4 shapes, fused: O = softmax(Q K^T / sqrt(128) on the band+global+Zipf mask) V, "
            "seq 16384, head 128, 32x32 blocks, Q/K/V ~ N(0,1)",
    "spgemm": "SpGEMM (bsr_matrix::spgemm): banded 16384x16384 BSR (32x32 blocks, half-width 32 blocks) "
              "times a second matrix of the same pattern",
    "spgemm_rand": "SpGEMM (bsr_matrix::spgemm): 16384x16384 BSR (32x32 blocks, uniform p=0.05) "
                   "times an independent matrix of the same shape and density",
}
DENSITIES = [0.01, 0.05, 0.10, 0.25, 0.50]
L2_FLUSH_BYTES = 256 << 20
REF_TOTAL_BUDGET_S = 150.0
WORKLOAD_SWEEP = WORKLOAD_DESC["sweep"]


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even float32 -> bf16 bits (finite inputs: the sum stays
    inside 32 bits)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    return ((u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)).astype(np.uint16)


def uniform_bf16(rng, shape, lo=-1.0, hi=1.0, chunk_rows=2048):
    """uniform[lo, hi) bf16 bits, generated in row chunks (bounded temporaries)."""
    out = np.empty(shape, dtype=np.uint16)
    flat = out.reshape(shape[0], -1)
    for r0 in range(0, shape[0], chunk_rows):
        r1 = min(shape[0], r0 + chunk_rows)
        x = rng.random((r1 - r0, flat.shape[1]), dtype=np.float32)
        x *= np.float32(hi - lo)
        x += np.float32(lo)
        flat[r0:r1] = f32_to_bf16(x)
    return out


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained"), "src": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "src": "fallback"}


# ------------------------------------------------------------- generators --
def _pattern_from_occupancy(occ):
    rp = np.concatenate([[0], np.cumsum(occ.sum(1))]).astype(np.int32)
    ci = np.nonzero(occ)[1].astype(np.int32)
    return rp, ci


def _pattern_from_sets(cols_per_row):
    counts = np.array([len(c) for c in cols_per_row], dtype=np.int64)
    rp = np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)
    ci = (np.concatenate([np.sort(np.asarray(c, dtype=np.int32)) for c in cols_per_row])
          if counts.sum() else np.zeros(0, np.int32))
    return rp, ci.astype(np.int32)


def gen_spmm_case(M, K, N, R, C, p, seed, name=None):
    rng = np.random.default_rng(seed)
    rp, ci = _pattern_from_occupancy(rng.random((M // R, K // C)) < p)
    vals = f32_to_bf16(rng.uniform(-1, 1, ci.size * R * C).astype(np.float32))
    B = f32_to_bf16(rng.uniform(-1, 1, (K, N)).astype(np.float32))
    return dict(kind="spmm", name=name or f"p={p}", M=M, K=K, N=N, R=R, C=C, p=p, rp=rp, ci=ci,
                vals=vals, B=B)


def gen_sddmm_case(M, N, K, R, C, p, seed, scale=1.0 / 16, name=None):
    """out = mask (.) (A @ B): A M x K, B K x N, mask M x N (pattern only)."""
    rng = np.random.default_rng(seed)
    rp, ci = _pattern_from_occupancy(rng.random((M // R, N // C)) < p)
    A = f32_to_bf16((rng.standard_normal((M, K)) * scale).astype(np.float32))
    B = f32_to_bf16((rng.standard_normal((K, N)) * scale).astype(np.float32))
    return dict(kind="sddmm", name=name or f"sddmm p={p}", M=M, N=N, K=K, R=R, C=C, p=p, rp=rp,
                ci=ci, mvals=None, A=A, B=B)


def gen_attention_mask(nb, rng, band=8, n_global=4, zipf_s=1.2, cap=64):
    """Block pattern of config 4: per block-row i the band i-4..i+3 (8 blocks),
    the first n_global block-columns, and min(Zipf(zipf_s), cap) further
    block-columns drawn uniformly without replacement."""
    lo, hi = -(band // 2), band // 2 - 1
    extra = np.minimum(rng.zipf(zipf_s, nb), cap)
    rows = []
    for i in range(nb):
        s = set(range(max(0, i + lo), min(nb, i + hi + 1)))
        s.update(range(min(n_global, nb)))
        want = int(min(extra[i], nb - len(s)))
        while want > 0:
            for c in rng.integers(0, nb, size=2 * want + 4):
                c = int(c)
                if c not in s:
                    s.add(c)
                    want -= 1
                    if want == 0:
                        break
        rows.append(sorted(s))
    return _pattern_from_sets(rows)


def gen_cfg4(seed, S=16384, D=128, R=32):
    rng = np.random.default_rng(seed)
    nb = S // R
    rp, ci = gen_attention_mask(nb, rng)
    Q = f32_to_bf16(rng.standard_normal((S, D)).astype(np.float32))
    Kt = f32_to_bf16(rng.standard_normal((D, S)).astype(np.float32))   # K^T, row-major D x S
    V = f32_to_bf16(rng.standard_normal((S, D)).astype(np.float32))
    # P: the mask's pattern with uniform[0,1] values normalised over each row
    nnzb = int(rp[-1])
    pv = rng.uniform(0, 1, (nnzb, R, R)).astype(np.float32)
    row_of_block = np.repeat(np.arange(nb), np.diff(rp))
    sums = np.zeros((nb, R), np.float64)
    np.add.at(sums, row_of_block, pv.sum(axis=2))
    pv /= sums[row_of_block][:, :, None].astype(np.float32)
    sddmm = dict(kind="sddmm", name="sddmm QK^T", M=S, N=S, K=D, R=R, C=R, p=None, rp=rp, ci=ci,
                 mvals=None, A=Q, B=Kt)
    spmm = dict(kind="spmm", name="spmm PV", M=S, K=S, N=D, R=R, C=R, p=None, rp=rp, ci=ci,
                vals=f32_to_bf16(pv.reshape(-1)), B=V)
    return [sddmm, spmm]


def gen_zipf_pattern(nbr, nbc, density, s, rng):
    """Power-law block-row counts (Zipf's law over ranks: the k-th heaviest
    block-row holds ~ A k^-s blocks, at most nbc, A set so that the mean
    density is `density`), rows in random order, column indices uniform
    without replacement."""
    w = np.arange(1, nbr + 1, dtype=np.float64) ** -s
    total = density * nbr * nbc
    lo, hi = 0.0, total
    for _ in range(100):                      # sum(min(nbc, A w)) is monotone in A
        mid = 0.5 * (lo + hi)
        if np.minimum(nbc, mid * w).sum() < total:
            lo = mid
        else:
            hi = mid
    counts = np.minimum(nbc, np.floor(hi * w)).astype(np.int64)
    short = int(round(total)) - int(counts.sum())
    for k in range(nbr):                      # hand out the rounding remainder
        if short <= 0:
            break
        if counts[k] < nbc:
            counts[k] += 1
            short -= 1
    counts = counts[rng.permutation(nbr)]
    rows = [rng.choice(nbc, size=int(c), replace=False) for c in counts]
    return _pattern_from_sets(rows)


def gen_cfg5(seed, M=65536, K=65536, N=8192, R=64, C=64, density=0.01, s=1.1):
    rng = np.random.default_rng(seed)
    rp, ci = gen_zipf_pattern(M // R, K // C, density, s, rng)
    vals = uniform_bf16(rng, (ci.size * R, C)).reshape(-1)
    B = uniform_bf16(rng, (K, N))
    return dict(kind="spmm", name="spmm cfg5", M=M, K=K, N=N, R=R, C=C, p=density, rp=rp, ci=ci,
                vals=vals, B=B)


def gen_spgemm_case(arp, aci, brp, bci, R, seed, name):
    """C = A @ B, both n x n blocks of R x R (uniform[-1, 1] values)."""
    rng = np.random.default_rng(seed)
    av = uniform_bf16(rng, (aci.size * R, R))
    bv = uniform_bf16(rng, (bci.size * R, R))
    nb = arp.size - 1
    pairs = int(np.diff(brp)[aci].sum())
    return dict(kind="spgemm", name=name, M=nb * R, K=nb * R, N=nb * R, R=R, C=R, Ra=R, Ca=R, Cb=R,
                rp=arp, ci=aci, vals=av, brp=brp, bci=bci, bvals=bv, pairs=pairs)


def gen_spgemm_band(seed, n=512, hw=32, R=32):
    rp, ci = _pattern_from_sets([np.arange(max(0, i - hw), min(n, i + hw + 1)) for i in range(n)])
    return gen_spgemm_case(rp, ci, rp, ci, R, seed, f"band hw{hw}")


def gen_spgemm_rand(seed, n=512, p=0.05, R=32):
    rng = np.random.default_rng(seed)
    arp, aci = _pattern_from_occupancy(rng.random((n, n)) < p)
    brp, bci = _pattern_from_occupancy(rng.random((n, n)) < p)
    return gen_spgemm_case(arp, aci, brp, bci, R, seed + 1, f"random p={p}")


def gen_attn(seed, S=16384, D=128, R=32):
    """Config 4's mask and shapes for the fused attention step."""
    rng = np.random.default_rng(seed)
    rp, ci = gen_attention_mask(S // R, rng)
    Q, K, V = (f32_to_bf16(rng.standard_normal((S, D)).astype(np.float32)) for _ in range(3))
    return dict(kind="attn", name="attention step", M=S, S=S, d=D, R=R, C=R, p=None, rp=rp, ci=ci,
                Q=Q, K=K, V=V, scale=1.0 / np.sqrt(D))


def workload_ops(workload, rank):
    """Host-side ops of one step of `workload` (rank picks the seed of the
    independent per-rank copies)."""
    base = 1234 + 1 + 100 * rank
    if workload == "sweep":
        return [gen_spmm_case(4096, 4096, 4096, 32, 32, p, base + i) for i, p in enumerate(DENSITIES)]
    if workload == "cfg1":
        return [gen_spmm_case(1024, 1024, 256, 32, 32, 0.10, base)]
    if workload == "cfg3":
        return [gen_sddmm_case(4096, 4096, 256, 32, 32, 0.05, base)]
    if workload == "cfg4":
        return gen_cfg4(base)
    if workload == "cfg5":
        return [gen_cfg5(1234)]   # one problem shared by all ranks
    if workload == "attn":
        return [gen_attn(base)]
    if workload == "spgemm":
        return [gen_spgemm_band(base)]
    if workload == "spgemm_rand":
        return [gen_spgemm_rand(base)]
    raise ValueError(workload)


def op_flops(op):
    """Effective FLOPs (reference formulas, GEMM_profiling/read_spmm_profiler.py:73
    and read_sddmm_profiler.py:75)."""
    nnzb = int(op["rp"][-1])
    if op["kind"] == "attn":
        # S = Q K^T on the mask's blocks and O = P V (the softmax is not counted)
        return 4.0 * nnzb * op["R"] * op["C"] * op["d"]
    if op["kind"] == "spgemm":
        return 2.0 * op["pairs"] * op["Ra"] * op["Ca"] * op["Cb"]
    if op["kind"] == "spmm":
        return 2.0 * nnzb * op["R"] * op["C"] * op["N"]
    return 2.0 * nnzb * op["R"] * op["C"] * op["K"] + nnzb * op["R"] * op["C"]


def spgemm_out_nnzb(op):
    """Block count of C (symbolic product of the patterns)."""
    nb = op["rp"].size - 1
    n = 0
    for i in range(nb):
        ks = op["ci"][op["rp"][i]:op["rp"][i + 1]]
        if ks.size:
            n += np.unique(np.concatenate([op["bci"][op["brp"][k]:op["brp"][k + 1]] for k in ks])).size
    return n


def op_bytes(op):
    """Algorithmic HBM bytes: every operand byte the result depends on, read
    once, plus the output written once."""
    nnzb = int(op["rp"][-1])
    R, C = op["R"], op["C"]
    if op["kind"] == "attn":
        return 4 * 2 * op["S"] * op["d"] + 4 * (nnzb + op["S"] // R + 1)
    if op["kind"] == "spgemm":
        if "out_nnzb" not in op:
            op["out_nnzb"] = spgemm_out_nnzb(op)
        nb_b = int(op["brp"][-1])
        return (2 * nnzb * op["Ra"] * op["Ca"] + 2 * nb_b * op["Ca"] * op["Cb"]
                + 2 * op["out_nnzb"] * op["Ra"] * op["Cb"] + 4 * (nnzb + nb_b + op["out_nnzb"]))
    ncols = np.unique(op["ci"]).size
    idx = 4 * (nnzb + op["M"] // R + 1)
    if op["kind"] == "spmm":
        return 2 * nnzb * R * C + idx + 2 * ncols * C * op["N"] + 2 * op["M"] * op["N"]
    nrows = int(np.count_nonzero(np.diff(op["rp"])))
    mask = 0 if op["mvals"] is None else 2 * nnzb * R * C
    return mask + idx + 2 * nrows * R * op["K"] + 2 * ncols * C * op["K"] + 2 * nnzb * R * C


# ---------------------------------------------------------------- clocks --
class ClockSampler:
    """SM clock and throttle reasons of the given GPUs, polled every 2 ms
    from a background thread through NVML (nvidia-smi as a fallback)."""
    NVML_REASONS = (("hw_slowdown", 0x8), ("sw_thermal_slowdown", 0x20),
                    ("hw_thermal_slowdown", 0x40), ("sw_power_cap", 0x4))

    def __init__(self, pci_locations, period_s=0.002):
        """pci_locations: (domain, bus, device) integers of each GPU to watch
        (torch's device properties); NVML handles are matched by enumeration."""
        self.rows = []
        self.stop_ev = threading.Event()
        self.thread = None
        self.smi = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            by_loc = {}
            for i in range(pynvml.nvmlDeviceGetCount()):
                h = pynvml.nvmlDeviceGetHandleByIndex(i)
                info = pynvml.nvmlDeviceGetPciInfo(h)
                by_loc[(int(info.domain), int(info.bus), int(info.device))] = h
            self.handles = [by_loc[tuple(int(v) for v in loc)] for loc in pci_locations]
            self.smax = max(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
                            for h in self.handles)
            self.thread = threading.Thread(target=self._poll, args=(period_s,), daemon=True)
            self.thread.start()
        except Exception:
            self.nv = None
            self._start_smi(",".join(f"{int(d):08X}:{int(b):02X}:{int(v):02X}.0"
                                     for d, b, v in pci_locations))

    def _poll(self, period):
        nv = self.nv
        while not self.stop_ev.is_set():
            for h in self.handles:
                try:
                    sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                    reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                    self.rows.append((float(sm), int(reasons)))
                except Exception:
                    pass
            self.stop_ev.wait(period)

    def _start_smi(self, bus_ids):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.fh = open(self.path, "w")
            self.smi = subprocess.Popen(
                ["nvidia-smi", "--query-gpu=clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,"
                 "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                 "clocks_event_reasons.sw_power_cap", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", bus_ids],
                stdout=self.fh, stderr=subprocess.DEVNULL)
        except Exception:
            self.smi = None

    def stop(self):
        if self.thread is not None:
            self.stop_ev.set()
            self.thread.join(timeout=5)
            if not self.rows:
                return None
            reasons = set()
            for _, bits in self.rows:
                for name, bit in self.NVML_REASONS:
                    if bits & bit:
                        reasons.add(name)
            return {"sm_mhz": float(np.median([r[0] for r in self.rows])),
                    "sm_max_mhz": float(self.smax), "reasons": sorted(reasons),
                    "samples": len(self.rows), "source": "nvml, 2 ms"}
        if self.smi is None:
            return None
        self.smi.terminate()
        try:
            self.smi.wait(timeout=5)
        except Exception:
            self.smi.kill()
        self.fh.close()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [x.strip() for x in line.split(",")]
                try:
                    rows.append((float(parts[0]), float(parts[1]), parts[2:6]))
                except (ValueError, IndexError):
                    continue
        os.unlink(self.path)
        if not rows:
            return None
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = {n for r in rows for n, v in zip(names, r[2]) if v.lower().startswith("active")}
        return {"sm_mhz": float(np.median([r[0] for r in rows])), "sm_max_mhz": rows[0][1],
                "reasons": sorted(reasons), "samples": len(rows), "source": "nvidia-smi, 100 ms"}


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


def reduce_over_ranks(x: float, dist, op="max") -> float:
    if dist is None:
        return x
    import torch

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX if op == "max" else dist.ReduceOp.SUM)
    return float(t.item())


def barrier(dist):
    import torch

    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()


# ------------------------------------------------------------ CPU baseline --
def _cpu_time(op, rows, threads, kind):
    """Seconds for the CPU golden (kind 'reference') or the oracle port over
    block-rows [0, rows) of `op`."""
    import oracle

    if op["kind"] == "attn":
        t0 = time.perf_counter()
        oracle.attention_bf16(op["rp"], op["ci"], op["S"], op["d"], op["Q"], op["K"], op["V"], op["scale"],
                              rows=(0, rows), use_ref=kind == "reference")
        return time.perf_counter() - t0
    if op["kind"] == "spgemm":
        # A's first `rows` block-rows times all of B (the reference's spgemm is one thread)
        arp = op["rp"][: rows + 1]
        n = int(arp[-1])
        aci, av = op["ci"][:n], op["vals"][: n * op["Ra"]]
        t0 = time.perf_counter()
        if kind == "reference":
            oracle.ref_spgemm_bf16(arp, aci, av, rows * op["Ra"], op["K"], op["Ra"], op["Ca"], op["brp"],
                                   op["bci"], op["bvals"], op["N"], op["Cb"])
        else:
            oracle.spgemm_bf16(arp, aci, av, op["Ra"], op["Ca"], op["brp"], op["bci"], op["bvals"],
                               op["Cb"], op["N"] // op["Cb"])
        return time.perf_counter() - t0
    if op["kind"] == "spmm":
        args = (op["rp"], op["ci"], op["vals"], op["M"], op["K"], op["R"], op["C"], op["B"], op["N"])
        if kind == "reference":
            return oracle.ref_spmm_timed(*args, (0, rows), threads)
        t0 = time.perf_counter()
        oracle.spmm_bf16(*args, threads=threads, rows=(0, rows))
        return time.perf_counter() - t0
    args = (op["rp"], op["ci"], op["mvals"], op["M"], op["N"], op["R"], op["C"], op["A"], op["B"],
            op["K"])
    if kind == "reference":
        return oracle.ref_sddmm_timed(*args, (0, rows), threads)
    t0 = time.perf_counter()
    oracle.sddmm_bf16(*args, threads=threads, rows=(0, rows))
    return time.perf_counter() - t0


def _sample_flops(op, rows):
    nnzb = int(op["rp"][rows])
    if op["kind"] == "attn":
        return 4.0 * nnzb * op["R"] * op["C"] * op["d"]
    if op["kind"] == "spgemm":
        return 2.0 * float(np.diff(op["brp"])[op["ci"][:nnzb]].sum()) * op["Ra"] * op["Ca"] * op["Cb"]
    if op["kind"] == "spmm":
        return 2.0 * nnzb * op["R"] * op["C"] * op["N"]
    return 2.0 * nnzb * op["R"] * op["C"] * op["K"] + nnzb * op["R"] * op["C"]


def cpu_calibrate(ops, budget_s=12.0, threads=None):
    """Per op, how many leading block-rows the CPU golden finishes in about
    budget_s / len(ops) seconds.  Returns (rows per op, kind)."""
    import oracle

    threads = threads or os.cpu_count() or 1
    kind = "reference" if oracle.ref_available() else "port"
    per_op = budget_s / len(ops)
    out = []
    for op in ops:
        nbr = op["M"] // op["R"]
        rows = min(max(threads, 1), nbr)
        for _ in range(8):
            t = _cpu_time(op, rows, threads, kind)
            if t >= per_op / 2 or rows >= nbr:
                break
            rows = min(nbr, int(rows * min(16.0, max(1.5, per_op / max(t, 1e-4)))))
        out.append(rows)
    return out, kind


def cpu_threads_used(ops, threads=None):
    """The reference's spgemm golden is a single-threaded loop; its SpMM and
    SDDMM goldens run on every host thread here."""
    if all(op["kind"] in ("spgemm", "attn") for op in ops):
        return 1
    return threads or os.cpu_count() or 1


def golden_name(ops):
    kinds = {op["kind"] for op in ops}
    names = {"spmm": "bsr_matrix::spmm_bfloat16", "sddmm": "bsr_matrix::sddmm",
             "spgemm": "bsr_matrix::spgemm",
             "attn": "bsr_matrix::sddmm (float) -> softmax (numpy) -> bsr_matrix::spmm_bfloat16"}
    return " / ".join(names[k] for k in sorted(kinds))


def cpu_sample_time(ops, rows, kind, threads=None):
    threads = threads or os.cpu_count() or 1
    f = t = 0.0
    desc = []
    for op, r in zip(ops, rows):
        t += _cpu_time(op, r, threads, kind)
        f += _sample_flops(op, r)
        desc.append(f"{op['name']}: {r}/{op['M'] // op['R']} block-rows")
    return f, t, "; ".join(desc)


# --------------------------------------------------------------- our arm --
class DevOp:
    """One op of the workload on the GPU: device operands, output, plan."""

    def __init__(self, op, dev, strategy, local):
        import torch

        import bsp

        self.op = op
        self.kind = op["kind"]
        if self.kind == "attn":
            S, d = op["S"], op["d"]
            self.mask = bsp.DeviceBSR.from_host(S, S, 32, 32, op["rp"], op["ci"], None, local)
            self.Q, self.K, self.V = (bsp.to_device_bf16(op[k], local).view(S, d) for k in ("Q", "K", "V"))
            self.out = torch.empty((S, d), dtype=torch.bfloat16, device="cuda")
            self.plan = bsp.AttnPlan(dev, self.mask, d)
        elif self.kind == "spgemm":
            self.A = bsp.DeviceBSR.from_host(op["M"], op["K"], op["Ra"], op["Ca"], op["rp"], op["ci"],
                                             op["vals"], local)
            self.Bm = bsp.DeviceBSR.from_host(op["K"], op["N"], op["Ca"], op["Cb"], op["brp"], op["bci"],
                                              op["bvals"], local)
            self.plan = bsp.SpgemmPlan(dev, self.A, self.Bm)
            op["out_nnzb"] = self.plan.nnzb
            self.out = torch.empty(max(self.plan.nnzb * op["Ra"] * op["Cb"], 8), dtype=torch.bfloat16,
                                   device="cuda")
        elif self.kind == "spmm":
            self.A = bsp.DeviceBSR.from_host(op["M"], op["K"], op["R"], op["C"], op["rp"], op["ci"],
                                             op["vals"], local)
            self.B = bsp.to_device_bf16(op["B"], local)
            self.out = torch.empty((op["M"], op["N"]), dtype=torch.bfloat16, device="cuda")
            self.plan = bsp.SpmmPlan(dev, self.A, op["N"], strategy)
        else:
            self.mask = bsp.DeviceBSR.from_host(op["M"], op["N"], op["R"], op["C"], op["rp"], op["ci"],
                                                op["mvals"], local)
            self.Ad = bsp.to_device_bf16(op["A"], local)
            self.Bd = bsp.to_device_bf16(op["B"], local)
            self.out = torch.empty(max(int(op["rp"][-1]) * op["R"] * op["C"], 8), dtype=torch.bfloat16,
                                   device="cuda")
            self.plan = bsp.SddmmPlan(dev, self.mask, op["K"], strategy)

    def run(self, stream):
        if self.kind == "attn":
            self.plan.execute(self.Q, self.K, self.V, self.out, self.op["scale"], stream)
        elif self.kind == "spgemm":
            self.plan.execute(self.A, self.Bm, self.out, stream)
        elif self.kind == "spmm":
            self.plan.execute(self.A, self.B, self.out, stream)
        else:
            self.plan.execute(self.mask, self.Ad, self.Bd, self.out, stream)

    def kernel(self):
        if self.kind == "attn":
            return "attn_tcgen05"
        if self.kind == "spgemm":
            return "spgemm_tcgen05"
        if self.kind == "sddmm":
            return "sddmm_rowstack_tcgen05" if self.plan.info().get("variant", 0) == 1 else "sddmm_bsr_tcgen05"
        return {1: "spmm_rowstack_tcgen05", 2: "spmm_pair_tcgen05", 3: "spmm_twin_tcgen05"}.get(
            self.plan.info().get("variant", 0), "spmm_bsr_tcgen05")

    def close(self):
        self.plan.close()


def strategy_for(op, name):
    """`--strategy auto`: DDA for SpMM (row-stacked: N = 256 MMAs, or N = 128
    tiles for a B of at most 128 columns; measured faster than the swap-AB SnF
    kernel on config 4's P V, 49 vs 74 us), CDA for SDDMM."""
    import bsp

    if name != "auto":
        return bsp.STRATEGIES[name]
    return bsp.DDA


SHARDED_WORKLOADS = ("sweep", "cfg1", "cfg3", "cfg4", "cfg5")


def is_sharded(workload, ws):
    """At N > 1 the BASELINE configs split ONE problem across the GPUs: SpMM
    output row-panels / SDDMM mask row-panels balanced by nonzero blocks."""
    return ws > 1 and workload in SHARDED_WORKLOADS


def _panel_op(op, br0, br1):
    """The host op restricted to block-rows [br0, br1) (for its byte count)."""
    rp = np.asarray(op["rp"], dtype=np.int64)
    d = dict(op)
    d["rp"] = (rp[br0:br1 + 1] - rp[br0]).astype(np.int32)
    d["ci"] = np.asarray(op["ci"])[rp[br0]:rp[br1]]
    d["M"] = (br1 - br0) * op["R"]
    return d


class ShardOp:
    """One op of the workload split over the ranks (this rank's panel)."""

    def __init__(self, op, dev, strategy, rank, ws, local):
        import torch

        import bsp
        import bsp_dist

        self.op, self.kind = op, op["kind"]
        if self.kind == "spmm":
            self.sh = bsp_dist.ShardedSpmm(dev, op["M"], op["K"], op["R"], op["C"], op["rp"], op["ci"], op["vals"],
                                           op["N"], rank, ws, strategy, fused=True)
            self.B = bsp.to_device_bf16(op["B"], local)
            self.out = torch.empty((op["M"], op["N"]), dtype=torch.bfloat16, device="cuda")
            self.sh.attach(self.out)   # collective: map the peers' copies of this C
            br0, br1 = int(self.sh.bounds[rank]), int(self.sh.bounds[rank + 1])
            self.kernel = "spmm_rowstack_tcgen05 / spmm_pair_tcgen05 (row panel)"
        else:
            self.sh = bsp_dist.ShardedSddmm(dev, op["M"], op["N"], op["K"], op["R"], op["C"], op["rp"], op["ci"],
                                            op["mvals"], rank, ws, strategy)
            self.A = bsp.to_device_bf16(op["A"], local)
            self.B = bsp.to_device_bf16(op["B"], local)
            self.out = torch.empty(max(int(op["rp"][-1]) * op["R"] * op["C"], 8), dtype=torch.bfloat16,
                                   device="cuda")
            br0, br1 = self.sh.br0, self.sh.br1
            self.kernel = "sddmm_rowstack_tcgen05 (mask row panel)"
        self.panel = _panel_op(op, br0, br1)
        self.flops = self.sh.flops
        self.bytes = op_bytes(self.panel) if br1 > br0 else 0

    def compute(self, stream):
        if self.kind == "spmm":
            self.sh.compute(self.B, self.out, stream)
        else:
            self.sh.compute(self.A, self.B, self.out, stream)

    def replicated(self, stream):
        if self.kind == "spmm":
            self.sh.run(self.B, self.out, stream, replicate=True, sync_before=False)
        else:
            self.sh.run(self.A, self.B, self.out, stream, replicate=True)

    def close(self):
        self.sh.close()


def run_bsp(args):
    import torch

    import bsp

    ws, rank, local = dist_env()
    dist = init_dist(ws, local)
    peaks = load_peaks()
    dev = bsp.device(local)
    stream = torch.cuda.current_stream()
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device="cuda")
    sharded = is_sharded(args.workload, ws)
    ops = workload_ops(args.workload, 0 if sharded else rank)   # one problem when sharded

    runs = []
    for op in ops:
        if sharded:
            so = ShardOp(op, dev, strategy_for(op, args.strategy), rank, ws, local)
            runs.append(dict(op=op, dev=so, flops=so.flops, bytes=so.bytes, times=[], rtimes=[],
                             name=op["name"], fn=so.compute, rfn=so.replicated, kernel=so.kernel))
        else:
            d = DevOp(op, dev, strategy_for(op, args.strategy), local)
            runs.append(dict(op=op, dev=d, flops=op_flops(op), bytes=op_bytes(op), times=[], name=op["name"],
                             fn=d.run, kernel=d.kernel(), plan=d.plan.info()))

    sync = torch.zeros(1, dtype=torch.float32, device="cuda") if dist is not None else None

    def step(record, key="times", fn="fn"):
        for r in runs:
            flush.zero_()
            if sync is not None and sharded:
                # line the ranks' streams up (outside the timed events): every
                # rank's op then starts together, no rank's time includes
                # waiting for a peer that is still flushing, and no rank
                # stores into a peer's C that the peer still reads
                dist.all_reduce(sync)
            if record:
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                e0.record(stream)
            r[fn](stream)
            if record:
                e1.record(stream)
                r[key].append((e0, e1))

    for _ in range(args.warmup):
        step(False)
    dev.synchronize()
    barrier(dist)
    sampler = None
    if rank == 0:
        devs = range(ws) if ws > 1 else [local]
        props = [torch.cuda.get_device_properties(i) for i in devs]
        sampler = ClockSampler([(p.pci_domain_id, p.pci_bus_id, p.pci_device_id) for p in props])
    for _ in range(args.steps):
        step(True)
    barrier(dist)
    clocks = sampler.stop() if sampler else None
    dev.synchronize()

    per = []
    total_t = total_f = 0.0
    for r in runs:
        ts = [a.elapsed_time(b) * 1e-3 for a, b in r["times"]]
        t = float(np.mean(ts))
        total_t += sum(ts)
        total_f += r["flops"] * len(ts)
        t_tc = r["flops"] / (peaks["bf16_tflops"] * 1e12)
        t_hbm = r["bytes"] / (peaks["hbm_gbs"] * 1e9)
        d = dict(name=r["name"], nnzb=int(r["op"]["rp"][-1]), ms=t * 1e3,
                 tflops=r["flops"] / t / 1e12, gbs=r["bytes"] / t / 1e9,
                 bound="tensor" if t_tc >= t_hbm else "hbm", roofline_frac=max(t_tc, t_hbm) / t)
        if "plan" in r:
            d["units"] = r["plan"].get("units")
        per.append(d)
    t_all = reduce_over_ranks(total_t, dist, "max")
    f_all = reduce_over_ranks(total_f, dist, "sum")
    value = f_all / t_all / 1e12

    replicated = None
    if sharded:
        # the same step with C replicated on every GPU: the SpMM epilogue
        # stores each C tile into every peer's C over NVLink (one small NCCL
        # all-reduce after the kernel marks completion); SDDMM panels travel
        # by NCCL send/receive
        for _ in range(max(1, args.warmup // 2)):
            step(False, fn="rfn")
        barrier(dist)
        for _ in range(args.steps):
            step(True, key="rtimes", fn="rfn")
        barrier(dist)
        rt = sum(a.elapsed_time(b) * 1e-3 for r in runs for a, b in r["rtimes"])
        rt = reduce_over_ranks(rt, dist, "max")
        replicated = {"value": f_all / rt / 1e12, "unit": "TFLOP/s", "ms_per_step": rt / args.steps * 1e3,
                      "exchange": "SpMM: C tiles stored into every peer's C by the kernel's epilogue over NVLink "
                                  "(CUDA IPC), one NCCL all-reduce per op; SDDMM: NCCL send/recv of block ranges"}

    # dominant launch = the op with the largest share of device time
    di = int(np.argmax([d["ms"] for d in per]))
    dom, dom_run = per[di], runs[di]
    if dom["bound"] == "tensor":
        roof = {"bound": "tensor", "achieved": dom["tflops"], "peak": peaks["bf16_tflops"],
                "unit": "TFLOP/s", "frac": dom["tflops"] / peaks["bf16_tflops"]}
    else:
        roof = {"bound": "hbm", "achieved": dom["gbs"], "peak": peaks["hbm_gbs"],
                "unit": "GB/s", "frac": dom["gbs"] / peaks["hbm_gbs"]}
    roof["traffic"] = traffic_for(args.workload, dom["name"]) if not sharded else None
    roof["peak_src"] = peaks["src"]
    roof["kernel"] = f"{dom_run['kernel']} ({dom['name']})"
    roof["algorithmic"] = dom_run["bytes"] if dom["bound"] == "hbm" else dom_run["flops"]

    e2e = run_e2e(args, runs, dev, dist, sharded, rank, ws)

    cpu = None
    if ws == 1 and not args.no_cpu:
        host_ops = [r["op"] for r in runs]
        rows, kind = cpu_calibrate(host_ops, budget_s=args.cpu_budget)
        f, t, sample = cpu_sample_time(host_ops, rows, kind)
        cpu = {"value": f / t / 1e12, "unit": "TFLOP/s", "cores": cpu_threads_used(host_ops),
               "kind": kind,
               "sample": sample + ("; reference golden " + golden_name(host_ops)
                                   if kind == "reference" else "; oracle restatement")}

    out = {
        "metric": METRICS[args.workload], "value": value, "unit": "TFLOP/s", "n_gpus": ws,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": t_all / args.steps * 1e3,
        "higher_is_better": True, "scaling": "strong" if sharded else "weak", "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded numpy, BASELINE config shapes and value distributions)",
        "config": bench_config(args, ws),
        "roofline": roof, "cpu_baseline": cpu, "e2e": e2e,
        "gpu_launches": args.steps * len(runs), "clocks": clocks, "per_op": per,
    }
    if replicated is not None:
        out["replicated"] = replicated
    if rank == 0:
        print(json.dumps(out), flush=True)
    for r in runs:
        r["dev"].close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def bench_config(args, ws):
    """The workload description both arms print (the same dict, so that the
    two lines name the same workload)."""
    return {"workload": WORKLOAD_DESC[args.workload], "name": args.workload,
            "strategy": args.strategy, "c_dtype": "bf16", "accumulate": "fp32",
            "l2": "flushed (256 MiB write) before every timed launch",
            "per_rank": ("row panels of one problem, balanced by nonzero blocks; C left row-sharded "
                         "(the replicated-C step is reported under 'replicated')"
                         if is_sharded(args.workload, ws) else "independent copy per rank") if ws > 1 else None}


def _pinned(a):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).pin_memory().numpy()


def run_e2e(args, runs, dev, dist, sharded, rank, ws):
    """The same metric end to end through the public C ABI with host buffers:
    every step copies the inputs in from pinned host memory and the results
    back.  SpMM ops go through one bsp_spmm_host_batch call per step (the
    jobs' copies in, kernels and copies out pipelined over the copy engines in
    both directions); SDDMM / attention / SpGEMM ops through their host-buffer
    calls.  Sharded (N > 1): each rank's jobs are its row panels (A panel and
    the whole B in, its C panel out)."""
    import torch

    import bsp

    steps = max(1, min(args.steps, args.e2e_steps))
    h2d = d2h = 0
    batch, others = [], []
    for r in runs:
        op = r["op"]
        src = r["dev"].panel if sharded else op
        if op["kind"] == "spmm":
            rp, ci = _pinned(src["rp"]), _pinned(src["ci"])
            b0 = int(np.asarray(op["rp"])[int(r["dev"].sh.bounds[rank])]) if sharded else 0
            R, C = op["R"], op["C"]
            vals = _pinned(np.asarray(op["vals"]).reshape(-1)[b0 * R * C:(b0 + int(rp[-1])) * R * C])
            job = dict(M=src["M"], K=op["K"], R=R, C=C, row_ptr=rp, col_idx=ci, values=vals, B=_pinned(op["B"]),
                       N=op["N"], out=torch.empty((src["M"], op["N"]), dtype=torch.int16).pin_memory()
                       .numpy().view(np.uint16))
            h2d += rp.nbytes + ci.nbytes + vals.nbytes + job["B"].nbytes
            d2h += job["out"].nbytes
            if src["M"] > 0:
                batch.append(job)
        elif op["kind"] == "sddmm":
            if sharded:
                sh = r["dev"].sh
                R = op["R"]
                A = _pinned(np.asarray(op["A"])[sh.br0 * R:sh.br1 * R])
                mv = None
            else:
                A, mv = _pinned(op["A"]), None
            rp, ci = _pinned(src["rp"]), _pinned(src["ci"])
            nv = int(rp[-1]) * op["R"] * op["C"]
            hc = dict(rp=rp, ci=ci, A=A, B=_pinned(op["B"]), M=src["M"],
                      out=torch.empty(max(nv, 1), dtype=torch.int16).pin_memory().numpy().view(np.uint16)[:nv])
            h2d += rp.nbytes + ci.nbytes + A.nbytes + hc["B"].nbytes
            d2h += hc["out"].nbytes
            if nv > 0:
                others.append((op, hc, mv))
        elif op["kind"] == "attn":
            hc = dict(rp=_pinned(op["rp"]), ci=_pinned(op["ci"]), Q=_pinned(op["Q"]), K=_pinned(op["K"]),
                      V=_pinned(op["V"]))
            h2d += sum(hc[k].nbytes for k in hc)
            d2h += 2 * op["S"] * op["d"]
            others.append((op, hc, None))
        else:
            hc = dict(rp=_pinned(op["rp"]), ci=_pinned(op["ci"]), v=_pinned(op["vals"]),
                      brp=_pinned(op["brp"]), bci=_pinned(op["bci"]), bv=_pinned(op["bvals"]))
            h2d += sum(hc[k].nbytes for k in hc)
            d2h += 4 * (op["M"] // op["Ra"] + 1) + op["out_nnzb"] * (4 + 2 * op["Ra"] * op["Cb"])
            others.append((op, hc, None))
    strat = bsp.STRATEGIES[args.strategy] if args.strategy != "auto" else bsp.DDA

    def one():
        if batch:
            bsp.spmm_host_batch(batch, strategy=strat, dev=dev)
        for op, hc, mv in others:
            if op["kind"] == "attn":
                bsp.attn_host(op["S"], op["d"], hc["rp"], hc["ci"], hc["Q"], hc["K"], hc["V"], op["scale"], dev=dev)
            elif op["kind"] == "spgemm":
                bsp.spgemm_host(op["M"], op["K"], op["N"], op["Ra"], op["Ca"], op["Cb"], hc["rp"], hc["ci"],
                                hc["v"], hc["brp"], hc["bci"], hc["bv"], dev=dev)
            else:
                bsp.sddmm_host(hc["M"], op["N"], op["R"], op["C"], hc["rp"], hc["ci"], mv, hc["A"], hc["B"],
                               op["K"], strategy=strat, dev=dev, out=hc["out"])

    one()  # warm (workspace growth, first touch of pinned pages)
    barrier(dist)
    t0 = time.perf_counter()
    for _ in range(steps):
        one()
    t = reduce_over_ranks(time.perf_counter() - t0, dist, "max")
    f = reduce_over_ranks(sum(r["flops"] for r in runs) * steps, dist, "sum")
    return {"value": f / t / 1e12, "unit": "TFLOP/s", "h2d_bytes_per_step": int(h2d),
            "d2h_bytes_per_step": int(d2h), "steps": steps,
            "path": ("bsp_spmm_host_batch (C ABI, host buffers: every SpMM of the step in one pipelined call)"
                     " / bsp_sddmm_host / bsp_attn_host / bsp_spgemm_host"
                     + ("; per rank: its row panels (A panel and all of B in, its C panel out)" if sharded
                        else ""))}


def traffic_for(workload, name):
    """DRAM bytes per launch of the dominant kernel from the committed ncu
    summary (profiles/traffic.json, keyed "<workload>:<op name>"), if one was
    captured for it."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return d.get(f"{workload}:{name}")
    except Exception:
        return None


# --------------------------------------------------------- reference arm --
def run_reference(args):
    """The reference arm: the reference's CPU golden on this box's host cores,
    the whole run (calibration, warm-up, timed steps) held to about
    REF_TOTAL_BUDGET_S seconds by the size of each step's block-row sample."""
    ws, rank, local = dist_env()
    if rank != 0:
        return
    ops = workload_ops(args.workload, 0)
    threads = os.cpu_count() or 1
    per_step = max(0.25, min(args.cpu_budget, REF_TOTAL_BUDGET_S / (args.steps + args.warmup + 2)))
    rows, kind = cpu_calibrate(ops, budget_s=per_step, threads=threads)
    sample = ""
    for _ in range(args.warmup):
        cpu_sample_time(ops, rows, kind, threads)
    tot_f = tot_t = 0.0
    for _ in range(args.steps):
        f, t, sample = cpu_sample_time(ops, rows, kind, threads)
        tot_f += f
        tot_t += t
    v = tot_f / tot_t / 1e12
    out = {"impl": "reference", "metric": METRICS[args.workload], "value": v, "unit": "TFLOP/s",
           "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
           "ms_per_step": tot_t / args.steps * 1e3, "higher_is_better": True,
           "scaling": "strong" if args.workload == "cfg5" else "weak", "vs_baseline": None,
           "dtype": "bf16", "data": "synthetic",
           "config": bench_config(args, ws),
           "cpu_baseline": {"value": v, "unit": "TFLOP/s", "cores": cpu_threads_used(ops, threads),
                            "kind": kind,
                            "sample": sample + ", every step"},
           "e2e": {"value": v, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)


# ---------------------------------------------------------------- ablation --
def table1_patterns():
    """The six cases of the reference's Table 1 (block_spmm/scripts/
    experiments_dram_reads_table.tex; M = N = K = 8192): Row R=C=256 d=25%,
    multi-diagonal R=C=256 d=50%, Row R=C=64 d=0.6%, multi-diagonal R=C=64
    d=0.6%, lower- and upper-triangular R=C=256.  Row fills the block grid in
    row-major order; multi-diagonal takes diagonals 0, +1, -1, +2, ... of the
    block grid (the reference generators' FILL_ROW / FILL_MULTI_DIAG /
    FILL_TRIL / FILL_TRIU)."""
    S = 8192

    def row_fill(nb, n):
        occ = np.zeros((nb, nb), bool)
        occ.flat[:n] = True
        return occ

    def multi_diag(nb, n):
        occ = np.zeros((nb, nb), bool)
        placed, d = 0, 0
        while placed < n:
            for t in range(nb):
                i, j = (t, t + d) if d >= 0 else (t - d, t)
                if i < nb and j < nb and placed < n:
                    occ[i, j] = True
                    placed += 1
            d = -d + 1 if d <= 0 else -d
        return occ

    out = []
    for name, R, occ in [("Row_R256_d25", 256, row_fill(32, 256)),
                         ("MultiDiag_R256_d50", 256, multi_diag(32, 512)),
                         ("Row_R64_d0.6", 64, row_fill(128, 98)),
                         ("MultiDiag_R64_d0.6", 64, multi_diag(128, 98)),
                         ("LowerTri_R256", 256, np.tril(np.ones((32, 32), bool))),
                         ("UpperTri_R256", 256, np.triu(np.ones((32, 32), bool)))]:
        rp, ci = _pattern_from_occupancy(occ)
        out.append((name, R, rp, ci, S))
    return out


def fig4_patterns():
    """The reference's Fig. 4 semi-sparse cases (paper_reproduce/reproduce_fig4.sh;
    block_spmm/inc/profiling_suite.hpp PatternD{5,10,25,50}[_128]): DDA at
    M = N = K = 8192 with R = C in {128, 256}, density d in {5, 10, 25, 50} %
    (round(d * blocks) blocks) and four fills: Row (row-major order), Col
    (column-major order), Multi-diag (diagonals 0, +1, -1, ...) and Random
    (seeded, distinct positions)."""
    S = 8192
    out = []
    for R in (128, 256):
        nb = S // R
        for d in (5, 10, 25, 50):
            n = max(1, int(round(nb * nb * d / 100.0)))
            occ_row = np.zeros((nb, nb), bool)
            occ_row.flat[:n] = True
            occ_col = np.zeros((nb, nb), bool)
            occ_col.T.flat[:n] = True
            occ_diag = np.zeros((nb, nb), bool)
            placed, dd = 0, 0
            while placed < n:
                for t in range(nb):
                    i, j = (t, t + dd) if dd >= 0 else (t - dd, t)
                    if i < nb and j < nb and placed < n:
                        occ_diag[i, j] = True
                        placed += 1
                dd = -dd + 1 if dd <= 0 else -dd
            rng = np.random.default_rng(5000 + R + d)
            occ_rand = np.zeros(nb * nb, bool)
            occ_rand[rng.choice(nb * nb, n, replace=False)] = True
            for pname, occ in (("Row", occ_row), ("Col", occ_col), ("MultiDiag", occ_diag),
                               ("Random", occ_rand.reshape(nb, nb))):
                rp, ci = _pattern_from_occupancy(occ)
                out.append((f"Fig4_{pname}_R{R}_d{d}", R, rp, ci, S))
    return out


def table3_cases():
    """The reference's Table 3 density sweep (block_sddmm/inc/profiling_suite.hpp
    SDDMMSweepDensity): SDDMM with M = N = K = 8192, R = C = 256 and a random
    mask of round(32 * 32 * d) blocks, d in {5, 10, 25, 50, 75} %."""
    S, R = 8192, 256
    nb = S // R
    out = []
    for d in (5, 10, 25, 50, 75):
        rng = np.random.default_rng(3000 + d)
        n = max(1, int(round(nb * nb * d / 100.0)))
        occ = np.zeros(nb * nb, bool)
        occ[rng.choice(nb * nb, n, replace=False)] = True
        rp, ci = _pattern_from_occupancy(occ.reshape(nb, nb))
        out.append((f"SDDMM_R256_d{d}", R, rp, ci, S))
    return out


def run_ablation_sddmm(args, dev, flush):
    """Table 3: SDDMM Naive / CDA / SnF (and their no-LB variants) on the
    reference's density sweep; effective FLOPs 2 nnzb R C K + nnzb R C."""
    import torch

    import bsp

    strategies = [("Naive", bsp.NAIVE, {}), ("CDA", bsp.DDA, {}), ("SnF", bsp.SNF, {}),
                  ("Naive_no_lb", bsp.NAIVE, dict(no_load_balance=1))]
    rng = np.random.default_rng(4321)
    A = B = None
    for name, R, rp, ci, S in table3_cases():
        if args.cases and not any(name.startswith(c) for c in args.cases.split(",")):
            continue
        if A is None:
            A = bsp.to_device_bf16(uniform_bf16(rng, (S, S)))
            B = bsp.to_device_bf16(uniform_bf16(rng, (S, S)))
        mask = bsp.DeviceBSR.from_host(S, S, R, R, rp, ci, None)
        out = torch.empty(ci.size * R * R, dtype=torch.bfloat16, device="cuda")
        flops = 2.0 * ci.size * R * R * S + ci.size * R * R
        for sname, strat, o in strategies:
            plan = bsp.SddmmPlan(dev, mask, S, strat, bsp.make_opts(**o))
            ts = []
            try:
                for it in range(args.warmup + args.steps):
                    flush.zero_()
                    e0 = torch.cuda.Event(enable_timing=True)
                    e1 = torch.cuda.Event(enable_timing=True)
                    e0.record()
                    plan.execute(mask, A, B, out)
                    e1.record()
                    torch.cuda.synchronize()
                    if it >= args.warmup:
                        ts.append(e0.elapsed_time(e1))
                dev.synchronize()
            except bsp.BspError as err:
                print(json.dumps({"case": name, "strategy": sname, "error": str(err)}), flush=True)
                plan.close()
                continue
            ms = float(np.median(ts))
            info = plan.info()
            print(json.dumps({"case": name, "strategy": sname, "R": R, "nnzb": int(ci.size), "K": S,
                              "units": info["units"], "keep_a": info["keep_a"], "ms": ms,
                              "tflops": flops / (ms * 1e-3) / 1e12}), flush=True)
            plan.close()


def run_ablation(args):
    """Per-strategy operand traffic and throughput on the Table 1 cases: the
    counterpart of the reference's count_dram_reads.py (in0 = A, in1 = B reads
    per core) and its *_no_lb variants.  One JSON line per (case, strategy):
    the bytes each plan moves with TMA (A, B, as multiples of reading each
    operand once), device time and effective TFLOP/s."""
    import torch

    import bsp

    dev = bsp.device(0)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device="cuda")
    strategies = [("Naive", bsp.NAIVE, {}), ("SnF", bsp.SNF, {}), ("DDA", bsp.DDA, {}),
                  ("Naive_no_lb", bsp.NAIVE, dict(no_load_balance=1)), ("SnF_no_lb", bsp.SNF, dict(no_load_balance=1)),
                  ("DDA_no_lb", bsp.DDA, dict(no_load_balance=1))]
    rng = np.random.default_rng(1234)
    run_ablation_sddmm(args, dev, flush)
    cases = [(c, strategies) for c in table1_patterns()]
    cases += [(c, [("DDA", bsp.DDA, {})]) for c in fig4_patterns()]  # Fig. 4 reports DDA only
    for (name, R, rp, ci, S), case_strategies in cases:
        if args.cases and not any(name.startswith(c) for c in args.cases.split(",")):
            continue
        vals = uniform_bf16(rng, (ci.size * R, R))
        B = uniform_bf16(rng, (S, S))
        A = bsp.DeviceBSR.from_host(S, S, R, R, rp, ci, vals)
        Bd = bsp.to_device_bf16(B)
        C = torch.empty((S, S), dtype=torch.bfloat16, device="cuda")
        flops = 2.0 * ci.size * R * R * S
        a_once = 2 * ci.size * R * R
        b_once = 2 * np.unique(ci).size * R * S
        for sname, strat, o in case_strategies:
            opts = bsp.make_opts(**o)
            tr = bsp.spmm_plan_traffic(S, S, R, R, rp, ci, S, strat, opts=opts, sm_count=dev.sm_count)
            plan = bsp.SpmmPlan(dev, A, S, strat, bsp.BF16, opts)
            ts = []
            try:
                for it in range(args.warmup + args.steps):
                    flush.zero_()
                    e0 = torch.cuda.Event(enable_timing=True)
                    e1 = torch.cuda.Event(enable_timing=True)
                    e0.record()
                    plan.execute(A, Bd, C)
                    e1.record()
                    torch.cuda.synchronize()
                    if it >= args.warmup:
                        ts.append(e0.elapsed_time(e1))
                dev.synchronize()
            except bsp.BspError as err:
                print(json.dumps({"case": name, "strategy": sname, "variant": tr["variant"], "error": str(err)}),
                      flush=True)
                plan.close()
                continue
            ms = float(np.median(ts))
            print(json.dumps({"case": name, "strategy": sname, "R": R, "nnzb": int(ci.size),
                              "variant": tr["variant"], "units": tr["units"],
                              "a_bytes": tr["a_bytes"], "b_bytes": tr["b_bytes"],
                              "a_boxes": tr["a_boxes"], "b_boxes": tr["b_boxes"],
                              "a_reads_x": tr["a_bytes"] / a_once, "b_reads_x": tr["b_bytes"] / b_once,
                              "ms": ms, "tflops": flops / (ms * 1e-3) / 1e12}), flush=True)
            plan.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="bsp", choices=["bsp", "reference"])
    ap.add_argument("--workload", default="sweep", choices=list(WORKLOAD_DESC))
    ap.add_argument("--strategy", default="auto", choices=["auto", "naive", "snf", "dda"])
    ap.add_argument("--cpu-budget", type=float, default=12.0)
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--nccl-exchange", action="store_true",
                    help="cfg5 with N > 1: exchange C panels by NCCL send/recv instead of the fused kernel")
    ap.add_argument("--ablation", action="store_true",
                    help="per-strategy TFLOP/s on the reference's Table 3 SDDMM density sweep and operand "
                         "traffic and TFLOP/s on its Table 1 SpMM cases")
    ap.add_argument("--cases", default="", help="--ablation: comma-separated case names or name prefixes")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.ablation:
        run_ablation(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_bsp(args)


if __name__ == "__main__":
    main()
