"""SpGEMM parity on the GPU: libbsp's tcgen05 kernel (through the C ABI) vs
the reference's bsr_matrix<T>::spgemm golden (committed fixtures) and the
CPU oracle (its bit-exact restatement).  Bar: C's pattern identical, values
within max relative error 1e-2 (bf16 in, fp32 accumulate, one bf16 rounding
per block in both)."""
import glob
import os

import numpy as np
import pytest

import oracle
from helpers import assert_bf16_close

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
FIXTURES = sorted(glob.glob(os.path.join(GOLDEN, "spgemm_*.npz")))


def rand_pattern(rng, nbr, nbc, p, empty_rows=(), repeats=0):
    rows = []
    for i in range(nbr):
        cols = [] if i in empty_rows else list(np.nonzero(rng.random(nbc) < p)[0])
        for _ in range(repeats):
            if cols:
                cols.append(cols[rng.integers(len(cols))])
        rng.shuffle(cols)
        rows.append(cols)
    rp = np.concatenate([[0], np.cumsum([len(r) for r in rows])]).astype(np.int32)
    ci = np.array([c for r in rows for c in r], dtype=np.int32)
    return rp, ci


def rand_vals(rng, n):
    return oracle.f32_to_bf16(rng.uniform(-1, 1, n).astype(np.float32))


def run_and_check(bsp, M, K, N, Ra, Ca, Cb, arp, aci, av, brp, bci, bv, gold=None, **opts):
    orp, oci, out = bsp.spgemm_host(M, K, N, Ra, Ca, Cb, arp, aci, av, brp, bci, bv,
                                    opts=bsp.make_opts(**opts))
    if gold is None:
        gold = oracle.spgemm_bf16(arp, aci, av, Ra, Ca, brp, bci, bv, Cb, N // Cb)
    assert np.array_equal(orp, gold[0]) and np.array_equal(oci, gold[1])
    assert_bf16_close(out, gold[2], what=f"spgemm {M}x{K}x{N} {Ra}/{Ca}/{Cb} {opts}")
    return orp, oci, out


@pytest.mark.parametrize("path", FIXTURES, ids=[os.path.basename(f)[:-4] for f in FIXTURES])
def test_spgemm_reference_fixtures(path):
    import bsp

    z = np.load(path)
    Ra, Ca, Cb = int(z["Ra"]), int(z["Ca"]), int(z["Cb"])
    run_and_check(bsp, int(z["Ha"]), int(z["Wa"]), int(z["Wb"]), Ra, Ca, Cb, z["a_indptr"],
                  z["a_indices"], z["a_values"], z["b_indptr"], z["b_indices"], z["b_values"],
                  gold=(z["out_indptr"], z["out_indices"], z["out"]))


BLOCKS = [(32, 32, 32), (64, 32, 32), (128, 32, 32), (32, 64, 32), (32, 128, 32), (32, 32, 64),
          (32, 32, 128), (64, 64, 64), (128, 128, 128), (64, 128, 32)]


@pytest.mark.parametrize("Ra,Ca,Cb", BLOCKS)
def test_spgemm_block_sizes(Ra, Ca, Cb):
    import bsp

    rng = np.random.default_rng(Ra + 3 * Ca + 11 * Cb)
    nbr, nbk, nbc = 23, 17, 29
    arp, aci = rand_pattern(rng, nbr, nbk, 0.2, empty_rows=(3,))
    brp, bci = rand_pattern(rng, nbk, nbc, 0.2, empty_rows=(0,))
    run_and_check(bsp, nbr * Ra, nbk * Ca, nbc * Cb, Ra, Ca, Cb, arp, aci,
                  rand_vals(rng, aci.size * Ra * Ca), brp, bci, rand_vals(rng, bci.size * Ca * Cb))


@pytest.mark.parametrize("opts", [dict(n_tiles=1), dict(n_tiles=2), dict(steps_per_stage=1),
                                  dict(steps_per_stage=4), dict(producers=1), dict(max_ctas=5),
                                  dict(no_load_balance=1), dict(no_load_balance=2)])
def test_spgemm_options(opts):
    import bsp

    rng = np.random.default_rng(17)
    arp, aci = rand_pattern(rng, 40, 30, 0.15)
    brp, bci = rand_pattern(rng, 30, 50, 0.15)
    run_and_check(bsp, 40 * 32, 30 * 32, 50 * 32, 32, 32, 32, arp, aci, rand_vals(rng, aci.size * 1024),
                  brp, bci, rand_vals(rng, bci.size * 1024), **opts)


@pytest.mark.parametrize("Ra,Ca,Cb", [(32, 32, 32), (64, 64, 32)])
def test_spgemm_repeated_columns(Ra, Ca, Cb):
    import bsp

    rng = np.random.default_rng(29)
    arp, aci = rand_pattern(rng, 13, 9, 0.3, repeats=3)
    brp, bci = rand_pattern(rng, 9, 11, 0.3, repeats=3)
    run_and_check(bsp, 13 * Ra, 9 * Ca, 11 * Cb, Ra, Ca, Cb, arp, aci, rand_vals(rng, aci.size * Ra * Ca),
                  brp, bci, rand_vals(rng, bci.size * Ca * Cb))


def test_spgemm_identity_is_exact():
    """Block-diagonal identity A: C's blocks are B's, bit for bit."""
    import bsp

    rng = np.random.default_rng(4)
    n = 37
    arp = np.arange(n + 1, dtype=np.int32)
    aci = np.arange(n, dtype=np.int32)
    av = oracle.f32_to_bf16(np.tile(np.eye(64, dtype=np.float32).ravel(), n))
    brp, bci = rand_pattern(rng, n, 21, 0.3)
    bv = rand_vals(rng, bci.size * 64 * 32)
    orp, oci, out = bsp.spgemm_host(n * 64, n * 64, 21 * 32, 64, 64, 32, arp, aci, av, brp, bci, bv)
    order = np.concatenate([np.argsort(bci[brp[i]:brp[i + 1]], kind="stable") + brp[i] for i in range(n)])
    assert np.array_equal(orp, brp) and np.array_equal(oci, bci[order])
    assert np.array_equal(out.reshape(-1, 64 * 32), bv.reshape(-1, 64 * 32)[order])


def test_spgemm_empty_product():
    import bsp

    arp = np.array([0, 1, 2], np.int32)
    aci = np.array([0, 0], np.int32)
    brp = np.array([0, 0, 1], np.int32)
    bci = np.array([1], np.int32)
    rng = np.random.default_rng(0)
    orp, oci, out = bsp.spgemm_host(64, 64, 64, 32, 32, 32, arp, aci, rand_vals(rng, 2048), brp, bci,
                                    rand_vals(rng, 1024))
    assert np.array_equal(orp, [0, 0, 0]) and oci.size == 0 and out.size == 0


def test_spgemm_device_api_and_plan_reuse():
    """SpgemmPlan on device-resident BSR: one plan, two value sets."""
    import bsp
    import torch

    rng = np.random.default_rng(8)
    M, K, N = 96 * 32, 64 * 32, 80 * 32
    arp, aci = rand_pattern(rng, M // 32, K // 32, 0.05)
    brp, bci = rand_pattern(rng, K // 32, N // 32, 0.05)
    dev = bsp.device(0)
    plan = None
    for trial in range(2):
        av, bv = rand_vals(rng, aci.size * 1024), rand_vals(rng, bci.size * 1024)
        A = bsp.DeviceBSR.from_host(M, K, 32, 32, arp, aci, av)
        B = bsp.DeviceBSR.from_host(K, N, 32, 32, brp, bci, bv)
        if plan is None:
            plan = bsp.SpgemmPlan(dev, A, B)
            info = plan.info()
            assert info["out_nnzb"] == plan.nnzb and info["units"] > 0
        out = torch.empty(plan.nnzb * 1024, dtype=torch.bfloat16, device="cuda")
        plan.execute(A, B, out)
        dev.synchronize()
        gold = oracle.spgemm_bf16(arp, aci, av, 32, 32, brp, bci, bv, 32, N // 32)
        assert np.array_equal(plan.row_ptr, gold[0]) and np.array_equal(plan.col_idx, gold[1])
        assert_bf16_close(bsp.to_host_bits(out), gold[2], what=f"plan reuse {trial}")
    C = bsp.spgemm(A, B)
    assert np.array_equal(C.h_row_ptr, gold[0])
    assert_bf16_close(bsp.to_host_bits(C.values)[: gold[2].size], gold[2], what="one-shot")
    plan.close()


def test_spgemm_mismatched_operands_raise():
    import bsp

    rng = np.random.default_rng(1)
    arp, aci = rand_pattern(rng, 4, 4, 0.5)
    brp, bci = rand_pattern(rng, 4, 4, 0.5)
    A = bsp.DeviceBSR.from_host(128, 128, 32, 32, arp, aci, rand_vals(rng, aci.size * 1024))
    B = bsp.DeviceBSR.from_host(128, 256, 32, 64, brp, bci, rand_vals(rng, bci.size * 2048))
    Bbad = bsp.DeviceBSR.from_host(256, 128, 64, 32, np.array([0, 0, 0, 0, 0], np.int32),
                                   np.zeros(0, np.int32), np.zeros(8, np.uint16))
    dev = bsp.device(0)
    with pytest.raises(bsp.BspError):
        bsp.SpgemmPlan(dev, A, Bbad)
    plan = bsp.SpgemmPlan(dev, A, B)
    with pytest.raises(bsp.BspError):
        plan.execute(B, A, None)
    plan.close()


@pytest.mark.parametrize("p", [0.02, 0.1])
def test_spgemm_large_vs_oracle(p):
    """4096-wide operands (oracle in C, a few seconds)."""
    import bsp

    rng = np.random.default_rng(int(p * 1000))
    n = 128
    arp, aci = rand_pattern(rng, n, n, p)
    brp, bci = rand_pattern(rng, n, n, p)
    run_and_check(bsp, n * 32, n * 32, n * 32, 32, 32, 32, arp, aci, rand_vals(rng, aci.size * 1024),
                  brp, bci, rand_vals(rng, bci.size * 1024))


def test_spgemm_banded_full_size_properties():
    """A banded 16384 x 16384 product (32 x 32 blocks): C = A @ A with A's band
    of half-width 3 has C's band of half-width 6; linearity in B (C(A, 2B) = 2
    C(A, B) exactly, since doubling is exact in bf16 and fp32) and a slab of
    rows checked against the oracle."""
    import bsp

    rng = np.random.default_rng(99)
    n = 512
    rows = [list(range(max(0, i - 3), min(n, i + 4))) for i in range(n)]
    rp = np.concatenate([[0], np.cumsum([len(r) for r in rows])]).astype(np.int32)
    ci = np.array([c for r in rows for c in r], np.int32)
    av = rand_vals(rng, ci.size * 1024)
    bv = rand_vals(rng, ci.size * 1024)
    M = n * 32
    orp, oci, out = bsp.spgemm_host(M, M, M, 32, 32, 32, rp, ci, av, rp, ci, bv)
    widths = np.diff(orp)
    assert widths.max() == 13 and widths.min() == 7
    bv2 = oracle.f32_to_bf16(oracle.bf16_to_f32(bv) * 2)
    _, _, out2 = bsp.spgemm_host(M, M, M, 32, 32, 32, rp, ci, av, rp, ci, bv2)
    assert np.array_equal(oracle.bf16_to_f32(out2), oracle.bf16_to_f32(out) * 2)
    # rows 100..131 (block-rows) against the oracle on a cut of A
    r0, r1 = 100, 132
    sub_rp = (rp[r0:r1 + 1] - rp[r0]).astype(np.int32)
    sub_ci = ci[rp[r0]:rp[r1]]
    sub_av = av[rp[r0] * 1024:rp[r1] * 1024]
    g = oracle.spgemm_bf16(sub_rp, sub_ci, sub_av, 32, 32, rp, ci, bv, 32, n)
    assert np.array_equal(oci[orp[r0]:orp[r1]], g[1])
    assert_bf16_close(out[orp[r0] * 1024:orp[r1] * 1024], g[2], what="banded slab")


def test_spgemm_c_abi_host_entry():
    """bsp_spgemm_host (size query, then the product, with launch timing)."""
    import bsp

    rng = np.random.default_rng(31)
    arp, aci = rand_pattern(rng, 30, 20, 0.2)
    brp, bci = rand_pattern(rng, 20, 25, 0.2)
    av, bv = rand_vals(rng, aci.size * 2048), rand_vals(rng, bci.size * 2048)
    orp, oci, out, ms = bsp.spgemm_host_c(30 * 64, 20 * 32, 25 * 64, 64, 32, 64, arp, aci, av, brp, bci,
                                          bv, iters=3)
    gold = oracle.spgemm_bf16(arp, aci, av, 64, 32, brp, bci, bv, 64, 25)
    assert np.array_equal(orp, gold[0]) and np.array_equal(oci, gold[1])
    assert_bf16_close(out, gold[2], what="C ABI host entry")
    assert ms > 0
