"""Multi-GPU BSR SpMM: output row-panels sharded across the GPUs of one node.

The reference runs on one Wormhole card and has no multi-device path; this is
the B200 scale-out of its SpMM (one process per GPU, torch.distributed for
the plumbing).  Block-rows of A are split into contiguous ranges with equal
nonzero-block counts (``bsp_partition_rows``: the reference's per-core
balancing criterion, block_spmm/inc/host_code/
bsr_spmm_multicore_load_balanced_new_DM.cpp:346-393, applied to GPU ranges
so that each GPU's C row-panel is contiguous).  Each rank multiplies its
panel of A by the whole (replicated) B into its rows of C; when the caller
needs the replicated C, the panels are exchanged with one grouped NCCL
send/receive per peer (an all-gather with unequal panel sizes, written
straight into the final C, no padding and no extra copies).

The exchange helpers here take any torch.distributed process group, so the
host logic runs under ``gloo`` on CPU tensors as well.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

import bsp


@dataclass
class RowPanel:
    """Block-rows [br0, br1) of a BSR matrix, re-based to start at row 0."""

    br0: int
    br1: int
    row_ptr: np.ndarray   # int32 [br1 - br0 + 1], starting at 0
    col_idx: np.ndarray   # int32 [nnzb of the panel]
    values: np.ndarray    # bf16 bits [nnzb * R * C] (or None)
    block0: int           # index of the panel's first block in the full matrix


def shard_bounds(row_ptr: np.ndarray, world_size: int) -> np.ndarray:
    """bounds[world_size + 1]: rank r owns block-rows [bounds[r], bounds[r+1])."""
    return bsp.partition_rows(np.asarray(row_ptr, dtype=np.int32), world_size)


def row_panel(row_ptr, col_idx, values, R: int, C: int, br0: int, br1: int) -> RowPanel:
    """Slice block-rows [br0, br1) out of a host BSR matrix (views, no copies
    of the block values beyond the slice)."""
    rp = np.asarray(row_ptr, dtype=np.int64)
    b0, b1 = int(rp[br0]), int(rp[br1])
    prp = (rp[br0:br1 + 1] - b0).astype(np.int32)
    pci = np.asarray(col_idx, dtype=np.int32)[b0:b1]
    pv = None
    if values is not None:
        pv = np.asarray(values, dtype=np.uint16).reshape(-1)[b0 * R * C:b1 * R * C]
    return RowPanel(br0, br1, prp, pci, pv, b0)


def exchange_row_panels(C_full, row_bounds, rank: int, world_size: int, group=None) -> None:
    """Replicate C across ranks: rank r holds rows [row_bounds[r], row_bounds[r+1])
    of ``C_full`` (a row-major 2-D tensor, the same shape on every rank) and
    receives every other rank's rows into place.  One grouped send/receive per
    peer; every rank issues the same set of operations in the same order."""
    import torch.distributed as dist

    if world_size == 1:
        return
    ops = []
    mine = C_full[int(row_bounds[rank]):int(row_bounds[rank + 1])]
    for peer in range(world_size):
        if peer == rank:
            continue
        theirs = C_full[int(row_bounds[peer]):int(row_bounds[peer + 1])]
        if mine.numel() > 0:
            ops.append(dist.P2POp(dist.isend, mine, peer, group))
        if theirs.numel() > 0:
            ops.append(dist.P2POp(dist.irecv, theirs, peer, group))
    if ops:
        for req in dist.batch_isend_irecv(ops):
            req.wait()


class ShardedSpmm:
    """C = A @ B with A's block-rows sharded over the ranks of ``group``.

    Every rank holds the whole B (K x N, bf16, on its GPU) and a full-size C;
    ``run`` computes this rank's row-panel with the single-GPU kernel and, if
    ``replicate``, exchanges panels so every rank ends with all of C.
    """

    def __init__(self, dev: "bsp.Device", M: int, K: int, R: int, C: int, row_ptr, col_idx,
                 values, N: int, rank: int, world_size: int, strategy=bsp.DDA, opts=None,
                 group=None):
        self.M, self.K, self.R, self.C, self.N = M, K, R, C, N
        self.rank, self.world_size, self.group = rank, world_size, group
        self.bounds = shard_bounds(row_ptr, world_size)
        br0, br1 = int(self.bounds[rank]), int(self.bounds[rank + 1])
        self.panel = row_panel(row_ptr, col_idx, values, R, C, br0, br1)
        self.row_bounds = self.bounds * R
        self.rows = (br1 - br0) * R
        self.A = None
        self.plan = None
        if self.rows > 0:
            self.A = bsp.DeviceBSR.from_host(self.rows, K, R, C, self.panel.row_ptr,
                                             self.panel.col_idx, self.panel.values,
                                             dev.ordinal)
            self.plan = bsp.SpmmPlan(dev, self.A, N, strategy, bsp.BF16, opts)

    @property
    def flops(self) -> float:
        """Effective FLOPs of this rank's panel (nonzero blocks only)."""
        return 2.0 * int(self.panel.row_ptr[-1]) * self.R * self.C * self.N

    def compute(self, B, C_full, stream=None) -> None:
        """This rank's panel only: C_full[panel rows] = A_panel @ B."""
        if self.plan is not None:
            r0 = int(self.row_bounds[self.rank])
            self.plan.execute(self.A, B, C_full[r0:r0 + self.rows], stream)

    def run(self, B, C_full, stream=None, replicate=True) -> None:
        self.compute(B, C_full, stream)
        if replicate:
            exchange_row_panels(C_full, self.row_bounds, self.rank, self.world_size, self.group)

    def close(self):
        if self.plan is not None:
            self.plan.close()
            self.plan = None
