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


def start_exchange(C_full, row_ranges, rank: int, world_size: int, group=None):
    """One exchange round: rank r owns rows row_ranges[r] = (r0, r1) of C_full
    (a row-major 2-D tensor, the same shape on every rank), sends them to every
    peer and receives every peer's range into place.  Every rank issues the
    same operations in the same order.  Returns the pending requests (the
    transfers run on the communicator's stream, after the work already queued
    on the current stream)."""
    import torch.distributed as dist

    if world_size == 1:
        return []
    ops = []
    r0, r1 = (int(v) for v in row_ranges[rank])
    mine = C_full[r0:r1]
    for peer in range(world_size):
        if peer == rank:
            continue
        p0, p1 = (int(v) for v in row_ranges[peer])
        theirs = C_full[p0:p1]
        if mine.numel() > 0:
            ops.append(dist.P2POp(dist.isend, mine, peer, group))
        if theirs.numel() > 0:
            ops.append(dist.P2POp(dist.irecv, theirs, peer, group))
    return dist.batch_isend_irecv(ops) if ops else []


def exchange_row_panels(C_full, row_bounds, rank: int, world_size: int, group=None) -> None:
    """Replicate C across ranks: rank r holds rows [row_bounds[r], row_bounds[r+1])
    and receives every other rank's rows into place (one round)."""
    ranges = [(row_bounds[r], row_bounds[r + 1]) for r in range(world_size)]
    for req in start_exchange(C_full, ranges, rank, world_size, group):
        req.wait()


def chunk_bounds(row_ptr, bounds, chunks: int) -> np.ndarray:
    """cb[r][c]: block-row bounds of chunk c of rank r's range (chunks of equal
    nonzero-block count, every rank cut into the same number of chunks)."""
    rp = np.asarray(row_ptr, dtype=np.int64)
    ws = len(bounds) - 1
    cb = np.zeros((ws, chunks + 1), dtype=np.int64)
    for r in range(ws):
        b0, b1 = int(bounds[r]), int(bounds[r + 1])
        if b1 > b0:
            sub = (rp[b0:b1 + 1] - rp[b0]).astype(np.int32)
            cb[r] = bsp.partition_rows(sub, chunks) + b0
        else:
            cb[r] = b0
    return cb


class ShardedSpmm:
    """C = A @ B with A's block-rows sharded over the ranks of ``group``.

    Every rank holds the whole B (K x N, bf16, on its GPU) and a full-size C;
    ``run`` computes this rank's row-panel with the single-GPU kernel and, if
    ``replicate``, makes every rank end with all of C.

    fused (default with more than one rank and a DDA plan): after ``attach(C)``
    (collective: the ranks map each other's C over NVLink), the kernel's
    epilogue stores every C tile into the local C and into each peer's C, so
    the all-gather rides along with the math, tile by tile; one small
    collective after the kernel tells every rank that all panels have landed.
    Otherwise the panels travel by NCCL send/receive: the panel is cut into
    ``chunks`` pieces of equal nonzero-block count and piece c crosses NVLink
    while piece c+1 is computed (``max_ctas``, default all SMs but 8, leaves
    SMs free for the communication kernels).
    """

    def __init__(self, dev: "bsp.Device", M: int, K: int, R: int, C: int, row_ptr, col_idx,
                 values, N: int, rank: int, world_size: int, strategy=bsp.DDA, opts=None,
                 group=None, chunks: int = None, max_ctas: int = None, fused: bool = None):
        self.M, self.K, self.R, self.C, self.N = M, K, R, C, N
        self.rank, self.world_size, self.group = rank, world_size, group
        self.dev = dev
        self.fused = (world_size > 1 and strategy == bsp.DDA) if fused is None else fused
        self.peer = None          # (bases, pointers) of the peers' C once attached
        self._sync = None
        self.bounds = shard_bounds(row_ptr, world_size)
        br0, br1 = int(self.bounds[rank]), int(self.bounds[rank + 1])
        self.panel = row_panel(row_ptr, col_idx, values, R, C, br0, br1)
        self.row_bounds = self.bounds * R
        self.rows = (br1 - br0) * R
        if chunks is None:
            chunks = 1 if (world_size == 1 or self.fused) else 4
        self.chunks = chunks
        self.cb = chunk_bounds(row_ptr, self.bounds, chunks)
        if opts is None and world_size > 1 and not self.fused:
            o = bsp.Opts()
            o.max_ctas = max_ctas if max_ctas is not None else max(1, dev.sm_count - 8)
            opts = o
        self.A = None       # the whole panel (one allocation)
        self.parts = []     # (row offset in C, DeviceBSR view, plan) per non-empty chunk
        if self.rows > 0:
            self.A = bsp.DeviceBSR.from_host(self.rows, K, R, C, self.panel.row_ptr,
                                             self.panel.col_idx, self.panel.values,
                                             dev.ordinal)
            for c in range(chunks):
                c0, c1 = int(self.cb[rank][c]), int(self.cb[rank][c + 1])
                if c1 <= c0:
                    self.parts.append(None)
                    continue
                sub = row_panel(row_ptr, col_idx, None, R, C, c0, c1)
                rows = (c1 - c0) * R
                rp_d = self.A.row_ptr[c0 - br0:c1 - br0 + 1] - int(self.panel.row_ptr[c0 - br0])
                blk0 = int(self.panel.row_ptr[c0 - br0])
                nblk = int(sub.row_ptr[-1])
                view = bsp.DeviceBSR(rows, K, R, C, rp_d.contiguous(),
                                     self.A.col_idx[blk0:blk0 + max(nblk, 1)],
                                     self.A.values[blk0 * R * C:(blk0 + max(nblk, 1)) * R * C]
                                     if self.A.values is not None else None,
                                     sub.row_ptr, sub.col_idx)
                plan = bsp.SpmmPlan(dev, view, N, strategy, bsp.BF16, opts)
                self.parts.append((c0 * R, view, plan))

    @property
    def flops(self) -> float:
        """Effective FLOPs of this rank's panel (nonzero blocks only)."""
        return 2.0 * int(self.panel.row_ptr[-1]) * self.R * self.C * self.N

    def _chunk_ranges(self, c):
        R = self.R
        return [(int(self.cb[r][c]) * R, int(self.cb[r][c + 1]) * R) for r in range(self.world_size)]

    def compute(self, B, C_full, stream=None) -> None:
        """This rank's panel only: C_full[panel rows] = A_panel @ B."""
        for part in self.parts:
            if part is not None:
                r0, view, plan = part
                plan.execute(view, B, C_full[r0:r0 + view.rows], stream)

    def attach(self, C_full) -> None:
        """Collective (every rank, same order): map every peer's C_full into
        this process so that the fused kernel can store into it."""
        import torch
        import torch.distributed as dist

        if not self.fused or self.world_size == 1:
            return
        self.detach()
        mine = bsp.ipc_export(self.dev, C_full)
        allh = [None] * self.world_size
        dist.all_gather_object(allh, mine, group=self.group)
        bases, ptrs = [], []
        for r in range(self.world_size):
            if r == self.rank:
                continue
            base = bsp.ipc_import(self.dev, allh[r][0])
            bases.append(base)
            ptrs.append(base + allh[r][1])
        self.peer = (bases, ptrs, C_full.data_ptr(), C_full.stride(0) * C_full.element_size())
        self._sync = torch.zeros(1, dtype=torch.float32, device=C_full.device)

    def detach(self) -> None:
        """Collective: unmap the peers' C (after every rank has stopped storing)."""
        import torch.distributed as dist

        if self.peer is None:
            return
        import torch

        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        for base in self.peer[0]:
            bsp.ipc_close(self.dev, base)
        self.peer = None

    def run(self, B, C_full, stream=None, replicate=True, sync_before=True) -> None:
        """sync_before (fused mode): one small collective first, so that no
        rank stores into a peer's C while that peer still reads its previous
        contents; a caller that already lines the ranks up passes False."""
        if not replicate or self.world_size == 1:
            self.compute(B, C_full, stream)
            return
        if self.fused:
            import torch
            import torch.distributed as dist

            if self.peer is None or self.peer[2] != C_full.data_ptr():
                raise RuntimeError("ShardedSpmm: attach(C_full) first (fused replication)")
            cur = torch.cuda.current_stream()
            if stream is not None and not isinstance(stream, torch.cuda.Stream):
                raise ValueError("ShardedSpmm.run (fused): pass a torch.cuda.Stream or None")
            s = cur if stream is None else stream
            # the collectives run on the current stream: order the kernels
            # after the first one and the second one after the kernels
            if sync_before:
                dist.all_reduce(self._sync, group=self.group)
            if s != cur:
                s.wait_stream(cur)
            row_bytes = self.peer[3]
            for part in self.parts:
                if part is not None:
                    r0, view, plan = part
                    plan.execute_replicated(view, B, C_full[r0:r0 + view.rows],
                                            [p + r0 * row_bytes for p in self.peer[1]], s)
            if s != cur:
                cur.wait_stream(s)
            dist.all_reduce(self._sync, group=self.group)   # every rank's stores have landed
            return
        reqs = []
        for c in range(self.chunks):
            part = self.parts[c] if c < len(self.parts) else None
            if part is not None:
                r0, view, plan = part
                plan.execute(view, B, C_full[r0:r0 + view.rows], stream)
            reqs += start_exchange(C_full, self._chunk_ranges(c), self.rank, self.world_size,
                                   self.group)
        for req in reqs:
            req.wait()

    def close(self):
        if self.peer is not None:
            self.detach()
        for part in self.parts:
            if part is not None:
                part[2].close()
        self.parts = []


class ShardedSddmm:
    """out = mask (.) (A @ B) with the mask's block-rows sharded over the ranks.

    The mask row-panels are split like the SpMM's (contiguous block-row ranges
    of equal nonzero-block count).  Rank r holds the whole B (K x N) and uses
    the rows of A of its panel; its output blocks are a contiguous range of the
    output (blocks are stored block-row by block-row), so ``compute`` writes
    straight into that range of a full-size output buffer.  ``run`` with
    ``replicate`` then exchanges the ranges by NCCL send/receive, so every rank
    ends with the whole output.
    """

    def __init__(self, dev: "bsp.Device", M: int, N: int, K: int, R: int, C: int, row_ptr, col_idx,
                 mask_values, rank: int, world_size: int, strategy=bsp.DDA, opts=None, group=None):
        self.M, self.N, self.K, self.R, self.C = M, N, K, R, C
        self.rank, self.world_size, self.group = rank, world_size, group
        rp = np.asarray(row_ptr, dtype=np.int64)
        self.bounds = shard_bounds(row_ptr, world_size)
        self.block_bounds = [int(rp[int(b)]) for b in self.bounds]
        br0, br1 = int(self.bounds[rank]), int(self.bounds[rank + 1])
        self.br0, self.br1 = br0, br1
        self.panel = row_panel(row_ptr, col_idx, mask_values, R, C, br0, br1)
        self.nnzb = int(self.panel.row_ptr[-1])
        self.mask = self.plan = None
        if self.nnzb > 0:
            self.mask = bsp.DeviceBSR.from_host((br1 - br0) * R, N, R, C, self.panel.row_ptr, self.panel.col_idx,
                                                self.panel.values, dev.ordinal)
            self.plan = bsp.SddmmPlan(dev, self.mask, K, strategy, opts)

    @property
    def flops(self) -> float:
        """Effective FLOPs of this rank's panel (the reference's SDDMM count)."""
        return 2.0 * self.nnzb * self.R * self.C * self.K + self.nnzb * self.R * self.C

    def compute(self, A_full, B, out_full, stream=None) -> None:
        """This rank's output blocks: out_full[blocks of the panel]."""
        if self.plan is None:
            return
        R, C = self.R, self.C
        b0, b1 = self.block_bounds[self.rank], self.block_bounds[self.rank + 1]
        self.plan.execute(self.mask, A_full[self.br0 * R:self.br1 * R], B, out_full[b0 * R * C:b1 * R * C], stream)

    def run(self, A_full, B, out_full, stream=None, replicate=True) -> None:
        self.compute(A_full, B, out_full, stream)
        if not replicate or self.world_size == 1:
            return
        blocks = out_full[:self.block_bounds[-1] * self.R * self.C].view(-1, self.R * self.C)
        ranges = [(self.block_bounds[r], self.block_bounds[r + 1]) for r in range(self.world_size)]
        for req in start_exchange(blocks, ranges, self.rank, self.world_size, self.group):
            req.wait()

    def close(self):
        if self.plan is not None:
            self.plan.close()
            self.plan = None
