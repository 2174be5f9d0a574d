"""GPU parity at the benchmark's own shapes, with the benchmark's own inputs
and plans (bench.py generators and strategy choice, rank 0 seeds):

* config 2, the headline density sweep: 4096^3, 32 x 32 blocks, every density,
  through the plan the benchmark times, compared with the oracle over all of
  C, and a relaunch of the same plan (split-K counters) giving the same bits;
* config 3 at its full 4096^2 size (SDDMM, every strategy);
* config 4 unfused at sequence 16384: the SDDMM Q K^T and the SpMM P V;
* config 5 (65536^2 with 64 x 64 blocks, Zipf rows, B 65536 x 8192) with the
  column-tile-order deal: the 16 heaviest and 48 random block-rows against
  the oracle, and the whole of C by its product with a random vector.

Bar: max relative error <= 1e-2 against the bf16 golden (helpers.TOL).
"""
import os
import sys
from concurrent.futures import ThreadPoolExecutor

import numpy as np
import pytest

import oracle
from helpers import TOL, assert_bf16_close

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
import bench  # noqa: E402  (the benchmark's generators)

pytestmark = pytest.mark.gpu

SEED0 = 1234 + 1   # bench.workload_ops(…, rank=0)


def _split_k_present(plan_info):
    return bool(((plan_info["unit_table"][:, 4] & 0xFF) > 1).any())


@pytest.mark.parametrize("i,p", list(enumerate(bench.DENSITIES)))
def test_config2_sweep_full_parity(i, p):
    import torch

    import bsp

    op = bench.gen_spmm_case(4096, 4096, 4096, 32, 32, p, SEED0 + i)
    M, K, N, R, C = op["M"], op["K"], op["N"], op["R"], op["C"]
    dev = bsp.device()
    strategy = bench.strategy_for(op, "auto")
    A = bsp.DeviceBSR.from_host(M, K, R, C, op["rp"], op["ci"], op["vals"])
    Bd = bsp.to_device_bf16(op["B"])
    plan = bsp.SpmmPlan(dev, A, N, strategy)
    info = plan.info()
    insp = bsp.inspect_spmm_plan(M, K, R, C, op["rp"], op["ci"], N, strategy, sm_count=dev.sm_count)
    assert insp["variant"] == info["variant"] and insp["units"] == info["units"]
    # the plan the benchmark times: CTA pairs from p = 0.25, single CTAs below;
    # split-K fills the balancer's last round at p = 0.25 and 0.5
    assert info["variant"] == (2 if p >= 0.25 else 1), info
    if p >= 0.25:
        assert _split_k_present(insp)
    gold = oracle.spmm_bf16(op["rp"], op["ci"], op["vals"], M, K, R, C, op["B"], N)
    outs = []
    for _ in range(2):
        Cd = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
        plan.execute(A, Bd, Cd)
        dev.synchronize()
        outs.append(bsp.to_host_bits(Cd))
    plan.close()
    assert np.array_equal(outs[0], outs[1])
    assert_bf16_close(outs[0], gold, tol=TOL, what=f"config 2 p={p}")


def test_config3_full_parity():
    import bsp

    op = bench.gen_sddmm_case(4096, 4096, 256, 32, 32, 0.05, SEED0)
    M, N, K, R, C = op["M"], op["N"], op["K"], op["R"], op["C"]
    gold = oracle.sddmm_bf16(op["rp"], op["ci"], None, M, N, R, C, op["A"], op["B"], K)
    for s in ("dda", "snf", "naive"):
        out = bsp.sddmm_host(M, N, R, C, op["rp"], op["ci"], None, op["A"], op["B"], K,
                             strategy=bsp.STRATEGIES[s])
        assert_bf16_close(out, gold, tol=TOL, what=f"config 3 {s}")


def test_config4_unfused_full_parity():
    import torch

    import bsp

    sd, sp = bench.gen_cfg4(SEED0)
    dev = bsp.device()
    # SDDMM Q K^T under the mask (the benchmark's strategy)
    S, D, R = sd["M"], sd["K"], sd["R"]
    mask = bsp.DeviceBSR.from_host(S, S, R, R, sd["rp"], sd["ci"], None)
    plan = bsp.SddmmPlan(dev, mask, D, bench.strategy_for(sd, "auto"))
    out = torch.empty(int(sd["rp"][-1]) * R * R, dtype=torch.bfloat16, device="cuda")
    plan.execute(mask, bsp.to_device_bf16(sd["A"]).view(S, D), bsp.to_device_bf16(sd["B"]).view(D, S), out)
    dev.synchronize()
    gold = oracle.sddmm_bf16(sd["rp"], sd["ci"], None, S, S, R, R, sd["A"], sd["B"], D)
    assert_bf16_close(bsp.to_host_bits(out), gold, tol=TOL, what="config 4 SDDMM")
    plan.close()
    # SpMM P V (P has the mask's pattern)
    A = bsp.DeviceBSR.from_host(S, S, R, R, sp["rp"], sp["ci"], sp["vals"])
    splan = bsp.SpmmPlan(dev, A, D, bench.strategy_for(sp, "auto"))
    Cd = torch.full((S, D), float("nan"), dtype=torch.bfloat16, device="cuda")
    splan.execute(A, bsp.to_device_bf16(sp["B"]).view(S, D), Cd)
    dev.synchronize()
    gold = oracle.spmm_bf16(sp["rp"], sp["ci"], sp["vals"], S, S, R, R, sp["B"], D)
    assert_bf16_close(bsp.to_host_bits(Cd), gold, tol=TOL, what="config 4 P V")
    splan.close()


def _rows_cols_oracle(rp, ci, vals, K, R, C, B, blocks, col_chunk):
    """Oracle of C[block-rows `blocks`], computed as independent (block-row,
    column chunk) pieces on host threads (the C oracle releases the GIL)."""
    vv = vals.reshape(-1, R * C)
    N = B.shape[1]
    out = np.zeros((len(blocks) * R, N), np.uint16)
    chunks = [(c0, min(N, c0 + col_chunk)) for c0 in range(0, N, col_chunk)]
    Bc = {c: np.ascontiguousarray(B[:, c[0]:c[1]]) for c in chunks}

    def one(job):
        k, b, c = job
        b0, b1 = int(rp[b]), int(rp[b + 1])
        g = oracle.spmm_bf16(np.array([0, b1 - b0], np.int32), ci[b0:b1], vv[b0:b1].reshape(-1), R, K, R, C,
                             Bc[c], c[1] - c[0], threads=1)
        out[k * R:(k + 1) * R, c[0]:c[1]] = g

    jobs = [(k, b, c) for k, b in enumerate(blocks) for c in chunks]
    with ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as ex:
        list(ex.map(one, jobs))
    return out


def test_config5_sampled_rows_and_whole_product():
    import torch

    import bsp

    op = bench.gen_cfg5(1234)
    M, K, N, R, C = op["M"], op["K"], op["N"], op["R"], op["C"]
    rp, ci = op["rp"], op["ci"]
    dev = bsp.device()
    A = bsp.DeviceBSR.from_host(M, K, R, C, rp, ci, op["vals"])
    Bd = bsp.to_device_bf16(op["B"])
    plan = bsp.SpmmPlan(dev, A, N, bench.strategy_for(op, "auto"))
    Cd = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
    plan.execute(A, Bd, Cd)
    dev.synchronize()
    plan.close()
    counts = np.diff(rp)
    heavy = np.argsort(-counts, kind="stable")[:16]
    rest = np.setdiff1d(np.arange(counts.size), heavy)
    rnd = np.random.default_rng(5).choice(rest, 48, replace=False)
    blocks = np.sort(np.concatenate([heavy, rnd]))
    gold = _rows_cols_oracle(rp, ci, op["vals"], K, R, C, op["B"], blocks, 1024)
    er = torch.from_numpy((blocks[:, None] * R + np.arange(R)[None, :]).reshape(-1)).cuda()
    got = bsp.to_host_bits(Cd.index_select(0, er))
    assert_bf16_close(got, gold, tol=TOL, what="config 5 sampled block-rows")
    # the whole of C: C v = A (B v) for a random sign vector v, relative to
    # || |C| |v| || (no cancellation in the scale)
    v = torch.from_numpy(np.random.default_rng(6).choice([-1.0, 1.0], N).astype(np.float32)).cuda()
    cv = (Cd.float() @ v).double().cpu().numpy()
    scale = np.linalg.norm(Cd.float().abs().sum(1).double().cpu().numpy())
    w = (Bd.float() @ v).double().cpu().numpy()
    y = np.zeros(M, np.float64)
    rows = np.repeat(np.arange(counts.size), counts)
    blk = oracle.bf16_to_f32(op["vals"]).reshape(-1, R, C)
    for s in range(0, ci.size, 2048):      # bounded temporaries
        contrib = np.einsum("brc,bc->br", blk[s:s + 2048].astype(np.float64), w.reshape(-1, C)[ci[s:s + 2048]])
        np.add.at(y.reshape(-1, R), rows[s:s + 2048], contrib)
    assert np.linalg.norm(cv - y) / scale <= 1e-2
