"""bsp_spmm_noalloc: the SpMM entry point that allocates no device memory.

It is for callers that cannot call cudaMalloc (device memory owned up front by
another allocator or pool).  Its scratch lives in a fixed array inside the
library, shared by every call, so this test calls it twice in a row with
different patterns and values and checks each result against the regular
entry point (bsp_spmm_plan_create + execute) within the parity tolerance.
The file sorts last so that a run stopping at the first failure has already
run every other test; it also passes on its own in a fresh process.
"""
import ctypes

import numpy as np
import pytest

from helpers import TOL, assert_bf16_close, rand_bsr, rand_dense

pytestmark = pytest.mark.gpu


def _noalloc(bsp, A, B, C, N, strategy):
    import torch

    d = A.desc()
    stream = torch.cuda.current_stream().cuda_stream
    st = bsp.lib().bsp_spmm_noalloc(ctypes.byref(d), A.h_row_ptr.ctypes.data, A.h_col_idx.ctypes.data,
                                    B.data_ptr(), B.stride(0), C.data_ptr(), C.stride(0), N, bsp.BF16,
                                    strategy, stream)
    if st != bsp.BSP_OK:
        raise bsp.BspError(st, bsp.lib().bsp_last_error_string().decode())


@pytest.mark.parametrize("strategy_name", ["naive", "snf"])
def test_noalloc_matches_regular_entry_point_twice(strategy_name):
    import torch

    import bsp

    strategy = bsp.STRATEGIES[strategy_name]
    cases = [(1024, 1024, 256, 32, 32, 0.10, 1), (512, 768, 384, 64, 32, 0.30, 2)]
    for M, K, N, R, C, p, seed in cases:  # two calls in a row through the shared scratch
        rng = np.random.default_rng(seed)
        rp, ci, vals = rand_bsr(rng, M, K, R, C, p, empty_rows=(1,))
        A = bsp.DeviceBSR.from_host(M, K, R, C, rp, ci, vals)
        B = bsp.to_device_bf16(rand_dense(rng, K, N))
        C_ref = bsp.spmm(A, B, strategy=strategy)  # the existing, allocating entry point
        C_na = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
        _noalloc(bsp, A, B, C_na, N, strategy)
        assert_bf16_close(bsp.to_host_bits(C_na), bsp.to_host_bits(C_ref), tol=TOL,
                          what=f"noalloc {strategy_name} {M}x{K}x{N}")


def test_noalloc_rejects_oversized_schedule_and_dda():
    import torch

    import bsp

    # DDA runs a different kernel: refused with a clear status
    M = K = 256
    rng = np.random.default_rng(3)
    rp, ci, vals = rand_bsr(rng, M, K, 32, 32, 0.5)
    A = bsp.DeviceBSR.from_host(M, K, 32, 32, rp, ci, vals)
    B = bsp.to_device_bf16(rand_dense(rng, K, 128))
    C = torch.empty((M, 128), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(bsp.BspError) as e:
        _noalloc(bsp, A, B, C, 128, bsp.DDA)
    assert e.value.status == bsp.BSP_ERR_UNSUPPORTED
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
    # the scratch is still usable after the refusals
    C3 = torch.full((M, 128), float("nan"), dtype=torch.bfloat16, device="cuda")
    _noalloc(bsp, A, B, C3, 128, bsp.SNF)
    assert_bf16_close(bsp.to_host_bits(C3), bsp.to_host_bits(bsp.spmm(A, B, strategy=bsp.SNF)), tol=TOL,
                      what="noalloc after refusal")
