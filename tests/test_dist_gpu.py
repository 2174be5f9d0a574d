"""Sharded SpMM and SDDMM on 2, 4 and 8 GPUs: row-panels by nonzero-block
count, replicated output.

Each rank runs the single-GPU kernel on its panel of A's (or the mask's)
block-rows and every rank ends with the whole output, either through the
fused SpMM kernel (the epilogue stores each tile into every GPU's C over
NVLink) or through NCCL send/receive of the panels; every rank's output must
match the oracle.  Each world size needs that many visible GPUs (skipped
otherwise).
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

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _case(kind="zipf"):
    import bench

    rng = np.random.default_rng(5)
    if kind == "skewed":
        # a few block-rows far longer than the rest: each rank's plan cuts
        # their units (split-K), and the merging part's stores reach both GPUs
        M, K, N, R, C = 4096, 8192, 256, 32, 32
        heavy = {3, 4, 5, 70, 71, 100}
        rows = [sorted(rng.choice(K // C, 230 if i in heavy else 5, replace=False)) for i in range(M // R)]
        rp = np.concatenate([[0], np.cumsum([len(r) for r in rows])]).astype(np.int32)
        ci = np.concatenate(rows).astype(np.int32)
    else:
        M = K = 2048
        N, R, C = 512, 64, 64
        rp, ci = bench.gen_zipf_pattern(M // R, K // C, 0.05, 1.1, rng)
    vals = bench.uniform_bf16(rng, (ci.size * R, C)).reshape(-1)
    B = bench.uniform_bf16(rng, (K, N))
    return M, K, N, R, C, rp, ci, vals, B


def _worker(rank, ws, port, q, fused, kind="zipf"):
    from datetime import timedelta

    import torch
    import torch.distributed as dist

    try:
        import bsp
        import bsp_dist
        import oracle
        from helpers import TOL, rel_err

        torch.cuda.set_device(rank)
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        dist.init_process_group("nccl", rank=rank, world_size=ws, timeout=timedelta(seconds=60),
                                device_id=torch.device("cuda", rank))
        M, K, N, R, C, rp, ci, vals, B = _case(kind)
        dev = bsp.device(rank)
        sh = bsp_dist.ShardedSpmm(dev, M, K, R, C, rp, ci, vals, N, rank, ws, bsp.DDA, fused=fused)
        Bd = bsp.to_device_bf16(B, rank)
        Cfull = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
        sh.attach(Cfull)
        for _ in range(2):   # twice: the second run overwrites the first
            sh.run(Bd, Cfull)
        torch.cuda.synchronize()
        dev.synchronize()
        got = oracle.bf16_to_f32(bsp.to_host_bits(Cfull).ravel())
        gold = oracle.bf16_to_f32(oracle.spmm_bf16(rp, ci, vals, M, K, R, C, B, N).ravel())
        err = float(rel_err(got, gold).max()) if np.all(np.isfinite(got)) else float("inf")
        sh.close()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, err <= TOL, err, sh.bounds.tolist()))
    except Exception as e:
        q.put((rank, False, repr(e), None))


def _spawn(target, ws, *args):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < ws:
        pytest.skip(f"needs {ws} visible GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, ws, port, q) + args) for r in range(ws)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(ws)]
    for p in procs:
        p.join(timeout=120)
    for rank, ok, err, bounds in res:
        assert ok, (rank, err)
    assert all(r[3] == res[0][3] for r in res)


@pytest.mark.parametrize("ws", [2, 4, 8])
@pytest.mark.parametrize("kind", ["zipf", "skewed"])
@pytest.mark.parametrize("fused", [True, False], ids=["fused-epilogue-stores", "nccl-send-recv"])
def test_sharded_spmm(ws, fused, kind):
    _spawn(_worker, ws, fused, kind)


def _sddmm_worker(rank, ws, port, q):
    from datetime import timedelta

    import torch
    import torch.distributed as dist

    try:
        import bench
        import bsp
        import bsp_dist
        import oracle
        from helpers import TOL, rel_err

        torch.cuda.set_device(rank)
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        dist.init_process_group("nccl", rank=rank, world_size=ws, timeout=timedelta(seconds=60),
                                device_id=torch.device("cuda", rank))
        op = bench.gen_sddmm_case(2048, 2048, 128, 32, 32, 0.1, 77)
        M, N, K, R, C = op["M"], op["N"], op["K"], op["R"], op["C"]
        dev = bsp.device(rank)
        sh = bsp_dist.ShardedSddmm(dev, M, N, K, R, C, op["rp"], op["ci"], None, rank, ws, bsp.DDA)
        A = bsp.to_device_bf16(op["A"], rank)
        B = bsp.to_device_bf16(op["B"], rank)
        out = torch.full((int(op["rp"][-1]) * R * C,), float("nan"), dtype=torch.bfloat16, device="cuda")
        for _ in range(2):
            sh.run(A, B, out)
        torch.cuda.synchronize()
        got = oracle.bf16_to_f32(bsp.to_host_bits(out))
        gold = oracle.bf16_to_f32(oracle.sddmm_bf16(op["rp"], op["ci"], None, M, N, R, C, op["A"], op["B"], K))
        err = float(rel_err(got, gold).max()) if np.all(np.isfinite(got)) else float("inf")
        sh.close()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, err <= TOL, err, sh.bounds.tolist()))
    except Exception as e:
        q.put((rank, False, repr(e), None))


@pytest.mark.parametrize("ws", [2, 4, 8])
def test_sharded_sddmm(ws):
    _spawn(_sddmm_worker, ws)
