"""Multi-GPU row-panel sharding, host side, on CPU with the gloo backend.

bsp_dist splits A's block-rows into contiguous ranges with equal nonzero-block
counts and exchanges the C row-panels with grouped send/receive.  Here two
(and three) ranks run as processes on CPU: each computes its own panel with
the oracle (standing in for the GPU kernel), the exchange runs over gloo, and
every rank must end with the full C, bit-identical to the oracle's one-shot
result.
"""
import os
import socket
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
PKG = os.path.join(ROOT, "tenstorrent-wh-blockspmm_b200")
for p in (ROOT, PKG, HERE):
    if p not in sys.path:
        sys.path.insert(0, p)

import bsp_dist  # noqa: E402
import oracle  # noqa: E402
from helpers import rand_bsr, rand_dense  # noqa: E402


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _case(seed, skew=False):
    rng = np.random.default_rng(seed)
    M, K, N, R, C = 512, 384, 96, 32, 32
    rp, ci, vals = rand_bsr(rng, M, K, R, C, 0.3, empty_rows=(2, 3))
    if skew:   # one heavy block-row and several empty ones
        occ = np.zeros((M // R, K // C), bool)
        occ[5, :] = True
        occ[0, ::3] = True
        occ[9, 1] = True
        rp = np.concatenate([[0], np.cumsum(occ.sum(1))]).astype(np.int32)
        ci = np.nonzero(occ)[1].astype(np.int32)
        vals = oracle.f32_to_bf16(rng.uniform(-1, 1, ci.size * R * C).astype(np.float32))
    B = rand_dense(rng, K, N)
    return M, K, N, R, C, rp, ci, vals, B


def _worker(rank, ws, port, seed, skew, q):
    import torch
    import torch.distributed as dist

    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=ws)
        M, K, N, R, C, rp, ci, vals, B = _case(seed, skew)
        bounds = bsp_dist.shard_bounds(rp, ws)
        panel = bsp_dist.row_panel(rp, ci, vals, R, C, int(bounds[rank]), int(bounds[rank + 1]))
        Cfull = torch.full((M, N), -1, dtype=torch.int16)   # stale data everywhere
        rows = (panel.br1 - panel.br0) * R
        if rows:
            part = oracle.spmm_bf16(panel.row_ptr, panel.col_idx, panel.values, rows, K, R, C, B, N)
            Cfull[panel.br0 * R:panel.br0 * R + rows] = torch.from_numpy(part.view(np.int16))
        bsp_dist.exchange_row_panels(Cfull, bounds * R, rank, ws)
        dist.barrier()
        full = oracle.spmm_bf16(rp, ci, vals, M, K, R, C, B, N)
        q.put((rank, bool(np.array_equal(Cfull.numpy().view(np.uint16), full)), bounds.tolist()))
        dist.destroy_process_group()
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, f"error: {e!r}", None))


def _chunk_worker(rank, ws, port, seed, chunks, q):
    """Chunked protocol: rank r computes chunk c of its panel, then round c of
    the exchange starts; all rounds are waited at the end."""
    import torch
    import torch.distributed as dist

    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=ws)
        M, K, N, R, C, rp, ci, vals, B = _case(seed)
        bounds = bsp_dist.shard_bounds(rp, ws)
        cb = bsp_dist.chunk_bounds(rp, bounds, chunks)
        assert cb[rank][0] == bounds[rank] and cb[rank][-1] == bounds[rank + 1]
        Cfull = torch.full((M, N), -1, dtype=torch.int16)
        reqs = []
        for c in range(chunks):
            c0, c1 = int(cb[rank][c]), int(cb[rank][c + 1])
            if c1 > c0:
                pan = bsp_dist.row_panel(rp, ci, vals, R, C, c0, c1)
                part = oracle.spmm_bf16(pan.row_ptr, pan.col_idx, pan.values, (c1 - c0) * R, K, R, C, B, N)
                Cfull[c0 * R:c1 * R] = torch.from_numpy(part.view(np.int16))
            ranges = [(int(cb[r][c]) * R, int(cb[r][c + 1]) * R) for r in range(ws)]
            reqs += bsp_dist.start_exchange(Cfull, ranges, rank, ws)
        for req in reqs:
            req.wait()
        dist.barrier()
        full = oracle.spmm_bf16(rp, ci, vals, M, K, R, C, B, N)
        q.put((rank, bool(np.array_equal(Cfull.numpy().view(np.uint16), full)), None))
        dist.destroy_process_group()
    except Exception as e:
        q.put((rank, f"error: {e!r}", None))


@pytest.mark.parametrize("ws,chunks", [(2, 3), (3, 4)])
def test_chunked_exchange_gloo(ws, chunks):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_chunk_worker, args=(r, ws, port, 21 + ws, chunks, q)) for r in range(ws)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(ws)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, ok, _ in results:
        assert ok is True, (rank, ok)


@pytest.mark.parametrize("ws,skew", [(2, False), (3, False), (2, True)])
def test_sharded_exchange_gloo(ws, skew):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, ws, port, 7 + ws, skew, q)) for r in range(ws)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(ws)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, ok, bounds in results:
        assert ok is True, (rank, ok)
    bounds = results[0][2]
    assert all(r[2] == bounds for r in results)


def test_shard_bounds_balance_and_cover():
    M, K, N, R, C, rp, ci, vals, B = _case(3)
    for ws in (1, 2, 3, 4, 8):
        b = bsp_dist.shard_bounds(rp, ws)
        assert b[0] == 0 and b[-1] == M // R and np.all(np.diff(b) >= 0)
        loads = np.diff(rp[b])
        # contiguous ranges can miss the ideal share by at most one block-row's blocks
        assert loads.max() - loads.min() <= 2 * np.diff(rp).max()


def test_row_panel_slices():
    M, K, N, R, C, rp, ci, vals, B = _case(4)
    p = bsp_dist.row_panel(rp, ci, vals, R, C, 3, 9)
    assert p.row_ptr[0] == 0 and p.row_ptr.size == 7
    assert np.array_equal(p.col_idx, ci[rp[3]:rp[9]])
    assert np.array_equal(p.values, vals[rp[3] * R * C:rp[9] * R * C])
    part = oracle.spmm_bf16(p.row_ptr, p.col_idx, p.values, 6 * R, K, R, C, B, N)
    full = oracle.spmm_bf16(rp, ci, vals, M, K, R, C, B, N)
    assert np.array_equal(part, full[3 * R:9 * R])
