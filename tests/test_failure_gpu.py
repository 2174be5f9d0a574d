"""Failure detection on the GPU without a fault: a bounded in-kernel wait is
made to run out (a pipeline stage that nothing fills), the launch gives up
through its drain path and reports BSP_ERR_TIMEOUT, and the device keeps
working; and split-K counts left behind by such a launch do not disturb the
launches after it.  These are the library's answer to the reference's hang
repros (block_spmm/inc/test_suite.hpp:72-73, block_sddmm/inc/test_suite.hpp:
112-171), whose device code could only hang."""
import ctypes

import numpy as np
import pytest

import oracle
from helpers import assert_bf16_close, rand_bsr, rand_dense

pytestmark = pytest.mark.gpu


def _skewed_rows(rng, nbr, nbc, heavy, heavy_len, light_len):
    rows = [sorted(rng.choice(nbc, heavy_len if i in heavy else light_len, replace=False)) for i in range(nbr)]
    rp = np.concatenate([[0], np.cumsum([len(r) for r in rows])]).astype(np.int32)
    return rp, np.concatenate(rows).astype(np.int32)


def test_bounded_wait_runs_out_then_device_recovers():
    import torch

    import bsp

    M = K = 2048
    N, R, C = 512, 32, 32
    rng = np.random.default_rng(77)
    rp, ci, vals = rand_bsr(rng, M, K, R, C, 0.2)
    B = rand_dense(rng, K, N)
    gold = oracle.spmm_bf16(rp, ci, vals, M, K, R, C, B, N)
    dev = bsp.device()
    A = bsp.DeviceBSR.from_host(M, K, R, C, rp, ci, vals)
    Bd = bsp.to_device_bf16(B)
    # single-CTA DDA kernel, 8 CTAs (so CTA 0 has many stages), 50 ms wait bound
    plan = bsp.SpmmPlan(dev, A, N, bsp.DDA, bsp.BF16, bsp.make_opts(group_mma=4, max_ctas=8, timeout_ms=50))
    assert plan.info()["variant"] == 1
    Cd = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
    # CTA 0 leaves its third stage unissued: the MMA warp's wait on it runs out
    bsp._check(bsp.lib().bsp_testing_spmm_drop_stage(plan.handle, 3))
    plan.execute(A, Bd, Cd)
    with pytest.raises(bsp.BspError) as e:
        dev.synchronize()
    assert e.value.status == bsp.BSP_ERR_TIMEOUT
    assert dev.status_bits() == 0          # read and cleared by the synchronize
    # the same plan, fault off, and a fresh plan: correct results, no error
    bsp._check(bsp.lib().bsp_testing_spmm_drop_stage(plan.handle, 0))
    for _ in range(2):
        Cd.fill_(float("nan"))
        plan.execute(A, Bd, Cd)
        dev.synchronize()
        assert_bf16_close(bsp.to_host_bits(Cd), gold, what="after a timed-out launch")
    plan.close()
    out = bsp.to_host_bits(bsp.spmm(A, Bd, strategy=bsp.DDA))
    assert_bf16_close(out, gold, what="fresh plan after a timed-out launch")


def _memset32(ptr, value, count):
    import torch

    torch.cuda.synchronize()
    cu = ctypes.CDLL("libcuda.so.1")
    cu.cuMemsetD32_v2.argtypes = [ctypes.c_uint64, ctypes.c_uint, ctypes.c_size_t]
    assert cu.cuMemsetD32_v2(ctypes.c_uint64(ptr), value, count) == 0
    torch.cuda.synchronize()


@pytest.mark.parametrize("variant", ["dda_1cta", "dda_pair"])
def test_split_k_counts_left_behind_do_not_disturb_later_launches(variant):
    """A launch that gives up mid-merge leaves its counter set non-zero.  The
    next launch uses the other set and zeroes this one, so both launches after
    it are exact (stands the left-behind counts in with a memset)."""
    import torch

    import bsp

    R = C = 32
    M, K, N = 4096, 8192, 256
    rng = np.random.default_rng(91)
    rp, ci = _skewed_rows(rng, M // R, K // C, heavy={3, 4, 5, 40, 41, 90}, heavy_len=230, light_len=5)
    vals = oracle.f32_to_bf16(rng.uniform(-1, 1, ci.size * R * C).astype(np.float32))
    B = rand_dense(rng, K, N)
    gold = oracle.spmm_bf16(rp, ci, vals, M, K, R, C, B, N)
    opts = bsp.make_opts(group_mma=4 if variant == "dda_1cta" else 5)
    A = bsp.DeviceBSR.from_host(M, K, R, C, rp, ci, vals)
    Bd = bsp.to_device_bf16(B)
    dev = bsp.device()
    plan = bsp.SpmmPlan(dev, A, N, bsp.DDA, bsp.BF16, opts)
    Cd = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
    plan.execute(A, Bd, Cd)
    dev.synchronize()
    ptr, per_set, nxt = ctypes.c_void_p(), ctypes.c_int64(), ctypes.c_int32()
    bsp._check(bsp.lib().bsp_testing_spmm_counters(plan.handle, ctypes.byref(ptr), ctypes.byref(per_set),
                                                   ctypes.byref(nxt)))
    assert ptr.value and per_set.value > 0 and nxt.value == 1
    # the set the first launch used (0) now holds counts as if it had given up
    _memset32(ptr.value, 3, per_set.value)
    for _ in range(3):
        Cd.fill_(float("nan"))
        plan.execute(A, Bd, Cd)
        dev.synchronize()
        assert_bf16_close(bsp.to_host_bits(Cd), gold, what=f"split-K {variant} after stale counts")
    plan.close()
