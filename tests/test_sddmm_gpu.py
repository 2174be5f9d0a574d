"""SDDMM parity on the GPU: libbsp (through the C ABI) vs the CPU oracle.

Cases mirror block_sddmm/inc/test_suite.hpp (single block, diagonal, full and
identity masks, nonsquare, R = C in {32, 64, 128, 256}, short K) plus
BASELINE config 3 scaled down.  Bar: max relative error <= 1e-2 vs the bf16
golden (restatement of bsr_matrix::sddmm) and the output pattern equal to
the mask's.
"""
import numpy as np
import pytest

import oracle
from helpers import assert_bf16_close, pcc, rand_bsr, rand_dense

pytestmark = pytest.mark.gpu

STRATS = ["naive", "dda", "snf"]

# (M, N, K, R, C, density, with_mask_values)
CASES = [
    (1024, 1024, 256, 32, 32, 0.05, False),   # BASELINE config 3 (scaled 1/4 per side)
    (512, 512, 256, 32, 32, 0.3, True),
    (256, 256, 128, 64, 64, 0.5, True),
    (256, 256, 128, 128, 128, 0.75, True),
    (512, 512, 256, 256, 256, 0.5, False),
    (256, 256, 96, 64, 32, 0.4, True),         # nonsquare, K = 96 (32-wide k chunks)
    (256, 384, 64, 32, 96, 0.4, True),         # C = 96: three segments per block
    (2048, 2048, 128, 32, 32, 0.02, False),    # attention-shaped: d = 128
    (128, 128, 32, 32, 32, 1.0, True),         # full mask, K = 32
    (1024, 256, 512, 512, 64, 0.5, True),      # R > 256: two slabs
]


# kernel variants: the row-stacked kernel (default; N = 256 or 128 MMAs) and
# the swap-AB kernel (one 4-segment unit per block-row slab, group_mma = 2)
KERNELS = {"rowstack": {}, "rowstack_n128": {"n_tiles": 1}, "swapab": {"group_mma": 2}}


def _run(bsp, M, N, K, R, C, rp, ci, mv, A, B, strategy, kernel="rowstack"):
    mask = bsp.DeviceBSR.from_host(M, N, R, C, rp, ci, mv)
    out = bsp.sddmm(mask, bsp.to_device_bf16(A), bsp.to_device_bf16(B),
                    strategy=bsp.STRATEGIES[strategy], opts=bsp.make_opts(**KERNELS[kernel]))
    return bsp.to_host_bits(out)


@pytest.mark.parametrize("case", CASES, ids=[f"{c[0]}x{c[1]}xK{c[2]}_R{c[3]}C{c[4]}_m{int(c[6])}" for c in CASES])
@pytest.mark.parametrize("strategy", STRATS)
@pytest.mark.parametrize("kernel", list(KERNELS))
def test_sddmm_parity(case, strategy, kernel):
    import bsp

    M, N, K, R, C, p, with_vals = case
    rng = np.random.default_rng(abs(hash((case, 2))) % 2**32)
    rp, ci, mv = rand_bsr(rng, M, N, R, C, p)
    if not with_vals:
        mv = None
    A = rand_dense(rng, M, K, "normal", 1 / 16)
    B = rand_dense(rng, K, N, "normal", 1 / 16)
    gold = oracle.sddmm_bf16(rp, ci, mv, M, N, R, C, A, B, K)
    out = _run(bsp, M, N, K, R, C, rp, ci, mv, A, B, strategy, kernel)
    assert_bf16_close(out, gold, what=f"{case} {strategy} {kernel}")
    if gold.size > 1:
        assert pcc(oracle.bf16_to_f32(out), oracle.bf16_to_f32(gold)) > 0.99


@pytest.mark.parametrize("kernel", list(KERNELS))
def test_sddmm_repeated_columns_and_partial_row_group(kernel):
    """A mask row naming one block-column twice gets both output blocks; 160
    rows leave the last 128-row group a quarter full."""
    import bsp

    M, N, K, R, C = 160, 256, 96, 32, 32
    rp = np.array([0, 3, 3, 5, 6, 8], np.int32)
    ci = np.array([2, 2, 5, 1, 1, 7, 0, 0], np.int32)
    rng = np.random.default_rng(11)
    mv = oracle.f32_to_bf16(rng.uniform(-2, 2, ci.size * R * C).astype(np.float32))
    A = rand_dense(rng, M, K, "normal", 1 / 8)
    B = rand_dense(rng, K, N, "normal", 1 / 8)
    gold = oracle.sddmm_bf16(rp, ci, mv, M, N, R, C, A, B, K)
    out = _run(bsp, M, N, K, R, C, rp, ci, mv, A, B, "naive", kernel)
    assert_bf16_close(out, gold, what=f"repeated columns {kernel}")


@pytest.mark.parametrize("strategy", STRATS)
def test_sddmm_host_api_keeps_pattern(strategy):
    import bsp

    M, N, K, R, C = 512, 512, 128, 32, 32
    rng = np.random.default_rng(77)
    rp, ci, mv = rand_bsr(rng, M, N, R, C, 0.2)
    A = rand_dense(rng, M, K, "normal", 1 / 16)
    B = rand_dense(rng, K, N, "normal", 1 / 16)
    gold = oracle.sddmm_bf16(rp, ci, mv, M, N, R, C, A, B, K)
    out = bsp.sddmm_host(M, N, R, C, rp, ci, mv, A, B, K, strategy=bsp.STRATEGIES[strategy])
    assert_bf16_close(out, gold)
    if oracle.ref_available():
        g2, oip, oix = oracle.ref_sddmm_bf16(rp, ci, mv, M, N, R, C, A, B, K)
        assert np.array_equal(oip, rp) and np.array_equal(oix, ci)
        assert np.array_equal(g2, gold)


def test_sddmm_empty_mask():
    import bsp
    import torch

    M, N, K, R, C = 256, 256, 64, 32, 32
    rp = np.zeros(M // R + 1, np.int32)
    mask = bsp.DeviceBSR.from_host(M, N, R, C, rp, np.zeros(0, np.int32), None)
    A = bsp.to_device_bf16(rand_dense(np.random.default_rng(0), M, K))
    B = bsp.to_device_bf16(rand_dense(np.random.default_rng(1), K, N))
    out = bsp.sddmm(mask, A, B)
    assert out.numel() == 0


def test_sddmm_identity_mask_known_answer():
    """block_sddmm/inc/test_suite.hpp test_identity_mask: mask blocks are
    identity matrices, so each output block is A*B restricted to its diagonal."""
    import bsp

    R = C = 32
    M = N = 4 * R
    K = 64
    rp = np.arange(5, dtype=np.int32)
    ci = np.arange(4, dtype=np.int32)
    eye = np.eye(R, dtype=np.float32)
    mv = oracle.f32_to_bf16(np.tile(eye.ravel(), 4))
    A = oracle.f32_to_bf16(np.arange(M * K, dtype=np.float32).reshape(M, K) / (M * K))
    B = oracle.f32_to_bf16(np.ones((K, N), np.float32))
    out = oracle.bf16_to_f32(_run(bsp, M, N, K, R, C, rp, ci, mv, A, B, "naive")).reshape(4, R, C)
    full = oracle.bf16_to_f32(A).astype(np.float64) @ oracle.bf16_to_f32(B).astype(np.float64)
    for b in range(4):
        expect = np.diag(np.diag(full[b * R:(b + 1) * R, b * C:(b + 1) * C]))
        np.testing.assert_allclose(out[b], expect, rtol=1e-2, atol=1e-6)


@pytest.mark.parametrize("K", [64, 128, 256])
@pytest.mark.parametrize("strategy", ["dda", "snf"])
def test_sddmm_resident_a_matches_streamed_a(K, strategy):
    """The resident-A kernel form (one A tile load per run of a row group's
    units) gives bit-identical output to the form that streams A with every
    stage (opts.group_rows = -1): same MMAs in the same order."""
    import bsp

    M, N, R, C = 2048, 4096, 32, 32
    rng = np.random.default_rng(K)
    rp, ci, mv = rand_bsr(rng, M, N, R, C, 0.15)
    Ah = rand_dense(rng, M, K, "normal", 1 / 16)
    Bh = rand_dense(rng, K, N, "normal", 1 / 16)
    A, B = bsp.to_device_bf16(Ah), bsp.to_device_bf16(Bh)
    mask = bsp.DeviceBSR.from_host(M, N, R, C, rp, ci, mv)
    outs = []
    # several producer warps loading A tiles (producers = 3, or N = 128 units
    # with a deep ring), with few CTAs so that each runs many row groups,
    # exercise the in-order issue and the final drain of the resident tiles
    for opts in (bsp.make_opts(group_rows=-1), bsp.make_opts(), bsp.make_opts(producers=3),
                 bsp.make_opts(n_tiles=1), bsp.make_opts(producers=3, max_ctas=7),
                 bsp.make_opts(n_tiles=1, max_ctas=5)):
        plan = bsp.SddmmPlan(bsp.device(), mask, K, bsp.STRATEGIES[strategy], opts)
        outs.append((plan.info()["keep_a"], bsp.to_host_bits(bsp.sddmm(mask, A, B, strategy=bsp.STRATEGIES[strategy], opts=opts))))
        plan.close()
    bsp.device().synchronize()
    assert [o[0] for o in outs] == [0, 1, 1, 1, 1, 1]
    for o in outs[1:]:
        assert np.array_equal(o[1], outs[0][1])
    gold = oracle.sddmm_bf16(rp, ci, mv, M, N, R, C, Ah, Bh, K)
    assert_bf16_close(outs[1][1], gold)
