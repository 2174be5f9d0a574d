"""bsp_spmm_noalloc: the SpMM entry point that allocates no device memory.

It is for callers that cannot call cudaMalloc (device memory owned up front by
another allocator or pool).  Its scratch lives in a fixed array inside the
library, shared by every call, so these tests call it twice in a row with
different patterns and values and check each result against the CPU oracle
(the restatement of the reference golden) and against the regular entry point
(bsp_spmm_plan_create + execute), for bf16 and f32 outputs.  The file sorts
last so that a run stopping at the first failure has already run every other
test; it also passes on its own in a fresh process.
"""
import ctypes

import numpy as np
import pytest

import oracle
from helpers import TOL, assert_bf16_close, normwise, rand_bsr, rand_dense

pytestmark = pytest.mark.gpu


def _noalloc(bsp, A, B, C, N, strategy, c_type=None):
    import torch

    d = A.desc()
    stream = torch.cuda.current_stream().cuda_stream
    st = bsp.lib().bsp_spmm_noalloc(ctypes.byref(d), A.h_row_ptr.ctypes.data, A.h_col_idx.ctypes.data,
                                    B.data_ptr(), B.stride(0), C.data_ptr(), C.stride(0), N,
                                    bsp.BF16 if c_type is None else c_type, strategy, stream)
    if st != bsp.BSP_OK:
        raise bsp.BspError(st, bsp.lib().bsp_last_error_string().decode())


CASES = [(1024, 1024, 256, 32, 32, 0.10, 1), (512, 768, 384, 64, 32, 0.30, 2)]


@pytest.mark.parametrize("strategy_name", ["naive", "snf"])
def test_noalloc_matches_oracle_and_regular_entry_point_twice(strategy_name):
    import torch

    import bsp

    strategy = bsp.STRATEGIES[strategy_name]
    for M, K, N, R, C, p, seed in CASES:  # two calls in a row through the shared scratch
        rng = np.random.default_rng(seed)
        rp, ci, vals = rand_bsr(rng, M, K, R, C, p, empty_rows=(1,))
        Bh = rand_dense(rng, K, N)
        A = bsp.DeviceBSR.from_host(M, K, R, C, rp, ci, vals)
        B = bsp.to_device_bf16(Bh)
        C_na = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
        _noalloc(bsp, A, B, C_na, N, strategy)
        out = bsp.to_host_bits(C_na)
        gold = oracle.spmm_bf16(rp, ci, vals, M, K, R, C, Bh, N)
        assert_bf16_close(out, gold, tol=TOL, what=f"noalloc {strategy_name} {M}x{K}x{N} vs oracle")
        C_ref = bsp.spmm(A, B, strategy=strategy)  # the existing, allocating entry point
        assert_bf16_close(out, bsp.to_host_bits(C_ref), tol=TOL,
                          what=f"noalloc {strategy_name} {M}x{K}x{N} vs bsp_spmm")


@pytest.mark.parametrize("strategy_name", ["naive", "snf"])
def test_noalloc_f32_output_twice(strategy_name):
    import torch

    import bsp

    strategy = bsp.STRATEGIES[strategy_name]
    for M, K, N, R, C, p, seed in CASES:
        rng = np.random.default_rng(100 + seed)
        rp, ci, vals = rand_bsr(rng, M, K, R, C, p, empty_rows=(2,))
        Bh = rand_dense(rng, K, N)
        A = bsp.DeviceBSR.from_host(M, K, R, C, rp, ci, vals)
        B = bsp.to_device_bf16(Bh)
        C_na = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
        _noalloc(bsp, A, B, C_na, N, strategy, c_type=bsp.F32)
        out = C_na.cpu().numpy()
        gold = oracle.spmm_f32(rp, ci, oracle.bf16_to_f32(vals), M, K, R, C, oracle.bf16_to_f32(Bh), N)
        assert np.all(np.isfinite(out))
        assert normwise(out, gold) <= 1e-5
        ref = bsp.spmm(A, B, strategy=strategy, c_type=bsp.F32).cpu().numpy()
        assert normwise(out, ref) <= 1e-5


def test_noalloc_rejects_bad_arguments_oversized_schedule_and_dda():
    import torch

    import bsp

    M = K = 256
    rng = np.random.default_rng(3)
    rp, ci, vals = rand_bsr(rng, M, K, 32, 32, 0.5)
    Bh = rand_dense(rng, K, 128)
    A = bsp.DeviceBSR.from_host(M, K, 32, 32, rp, ci, vals)
    B = bsp.to_device_bf16(Bh)
    C = torch.empty((M, 128), dtype=torch.bfloat16, device="cuda")
    # DDA runs a different kernel: refused with a clear status
    with pytest.raises(bsp.BspError) as e:
        _noalloc(bsp, A, B, C, 128, bsp.DDA)
    assert e.value.status == bsp.BSP_ERR_UNSUPPORTED
    # an output type other than bf16 / f32 is refused before any launch
    with pytest.raises(bsp.BspError) as e:
        _noalloc(bsp, A, B, C, 128, bsp.SNF, c_type=7)
    assert e.value.status == bsp.BSP_ERR_INVALID_ARG
    # block values not 16-byte aligned are refused
    shifted = bsp.DeviceBSR(A.rows, A.cols, A.R, A.C, A.row_ptr, A.col_idx, A.values[1:],
                            A.h_row_ptr, A.h_col_idx)
    with pytest.raises(bsp.BspError) as e:
        _noalloc(bsp, shifted, B, C, 128, bsp.SNF)
    assert e.value.status == bsp.BSP_ERR_INVALID_ARG
    # A schedule larger than the fixed scratch is refused before any launch.
    # An empty 163840 x 32 matrix times 32 x 4096 still has one unit per
    # 32-row block x 128-column tile: 163840 units of 32 bytes = 5 MiB.  The
    # operands are full size, so the call would be valid if it were accepted.
    M2, K2, N2 = 163840, 32, 4096
    rp2 = np.zeros(M2 // 32 + 1, np.int32)
    plan = bsp.inspect_spmm_plan(M2, K2, 32, 32, rp2, np.zeros(0, np.int32), N2, strategy=bsp.NAIVE)
    assert plan["units"] * 32 > 4 << 20
    A2 = bsp.DeviceBSR.from_host(M2, K2, 32, 32, rp2, np.zeros(0, np.int32), np.zeros(0, np.uint16))
    B2 = torch.zeros((K2, N2), dtype=torch.bfloat16, device="cuda")
    C2 = torch.empty((M2, N2), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(bsp.BspError) as e:
        _noalloc(bsp, A2, B2, C2, N2, bsp.NAIVE)
    assert e.value.status == bsp.BSP_ERR_UNSUPPORTED
    assert "scratch" in str(e.value)
    del C2
    # the scratch is still usable after the refusals, and gives the oracle's result
    C3 = torch.full((M, 128), float("nan"), dtype=torch.bfloat16, device="cuda")
    _noalloc(bsp, A, B, C3, 128, bsp.SNF)
    assert_bf16_close(bsp.to_host_bits(C3), oracle.spmm_bf16(rp, ci, vals, M, K, 32, 32, Bh, 128), tol=TOL,
                      what="noalloc after refusal")
