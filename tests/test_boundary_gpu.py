"""The C ABI's storage entry points on the GPU: bsp_bsr_upload / bsp_bsr_free
(a persistent device BSR for any number of plans) and the buffer helpers
(bsp_buffer_alloc / write / read / free, the reference's MakeBuffer and
EnqueueWrite/ReadBuffer), driven through ctypes exactly as a C caller would."""
import ctypes

import numpy as np
import pytest

import oracle
from helpers import assert_bf16_close, rand_bsr, rand_dense

pytestmark = pytest.mark.gpu


def _buf(bsp, dev, nbytes):
    p = ctypes.c_void_p()
    bsp._check(bsp.lib().bsp_buffer_alloc(dev.handle, nbytes, ctypes.byref(p)))
    return p.value


@pytest.mark.parametrize("strategy", ["naive", "snf", "dda"])
def test_bsr_upload_buffers_execute_free(strategy):
    import bsp

    dev = bsp.device()
    L = bsp.lib()
    M, K, N, R, C = 1024, 768, 384, 32, 32
    rng = np.random.default_rng(17)
    rp, ci, vals = rand_bsr(rng, M, K, R, C, 0.2, empty_rows=(0, 5))
    B = rand_dense(rng, K, N)
    gold = oracle.spmm_bf16(rp, ci, vals, M, K, R, C, B, N)
    desc = bsp.BsrDesc()
    bsp._check(L.bsp_bsr_upload(dev.handle, M, K, R, C, int(rp[-1]), rp.ctypes.data, ci.ctypes.data,
                                vals.ctypes.data, ctypes.byref(desc)))
    assert desc.values % 256 == 0 and desc.col_idx % 256 == 0 and desc.nnzb == int(rp[-1])
    dB, dC = _buf(bsp, dev, B.nbytes), _buf(bsp, dev, M * N * 2)
    bsp._check(L.bsp_buffer_write(dev.handle, dB, B.ctypes.data, B.nbytes))
    plan = ctypes.c_void_p()
    bsp._check(L.bsp_spmm_plan_create(dev.handle, ctypes.byref(desc), None, None, N, bsp.BF16,
                                      bsp.STRATEGIES[strategy], None, ctypes.byref(plan)))
    out = np.zeros((M, N), np.uint16)
    for _ in range(2):
        bsp._check(L.bsp_spmm_execute(plan, ctypes.byref(desc), dB, N, dC, N, None))
        bsp._check(L.bsp_device_synchronize(dev.handle))
        bsp._check(L.bsp_buffer_read(dev.handle, out.ctypes.data, dC, out.nbytes))
        assert_bf16_close(out, gold, what=f"upload + buffers {strategy}")
    bsp._check(L.bsp_spmm_plan_destroy(plan))
    bsp._check(L.bsp_buffer_free(dev.handle, dB))
    bsp._check(L.bsp_buffer_free(dev.handle, dC))
    bsp._check(L.bsp_bsr_free(dev.handle, ctypes.byref(desc)))
    assert desc.row_ptr is None and desc.values is None and desc.nnzb == 0


def test_bsr_upload_pattern_only_mask_and_rejects_bad_patterns():
    import bsp

    dev = bsp.device()
    L = bsp.lib()
    M, N, Kd, R = 512, 512, 64, 32
    rng = np.random.default_rng(19)
    rp, ci, _ = rand_bsr(rng, M, N, R, R, 0.25)
    desc = bsp.BsrDesc()
    bsp._check(L.bsp_bsr_upload(dev.handle, M, N, R, R, int(rp[-1]), rp.ctypes.data, ci.ctypes.data, None,
                                ctypes.byref(desc)))
    assert desc.values is None
    A = rand_dense(rng, M, Kd)
    Bm = rand_dense(rng, Kd, N)
    dA, dB = _buf(bsp, dev, A.nbytes), _buf(bsp, dev, Bm.nbytes)
    dO = _buf(bsp, dev, int(rp[-1]) * R * R * 2)
    bsp._check(L.bsp_buffer_write(dev.handle, dA, A.ctypes.data, A.nbytes))
    bsp._check(L.bsp_buffer_write(dev.handle, dB, Bm.ctypes.data, Bm.nbytes))
    bsp._check(L.bsp_sddmm(dev.handle, ctypes.byref(desc), dA, Kd, dB, N, Kd, dO, bsp.DDA, None, None))
    out = np.zeros(int(rp[-1]) * R * R, np.uint16)
    bsp._check(L.bsp_buffer_read(dev.handle, out.ctypes.data, dO, out.nbytes))
    assert_bf16_close(out, oracle.sddmm_bf16(rp, ci, None, M, N, R, R, A, Bm, Kd), what="upload mask sddmm")
    for p in (dA, dB, dO):
        bsp._check(L.bsp_buffer_free(dev.handle, p))
    bsp._check(L.bsp_bsr_free(dev.handle, ctypes.byref(desc)))
    # bad patterns are refused before any allocation
    bad_rp = rp.copy()
    bad_rp[3], bad_rp[4] = bad_rp[4], bad_rp[3] - 1
    bad_ci = ci.copy()
    bad_ci[0] = N // R
    for r_, c_ in ((bad_rp, ci), (rp, bad_ci)):
        st = L.bsp_bsr_upload(dev.handle, M, N, R, R, int(rp[-1]), r_.ctypes.data, c_.ctypes.data, None,
                              ctypes.byref(desc))
        assert st == bsp.BSP_ERR_INVALID_ARG and desc.row_ptr is None


@pytest.mark.parametrize("strategy", ["naive", "dda"])
def test_spmm_host_batch_matches_oracle(strategy):
    """bsp_spmm_host_batch: several products of different shapes, block sizes
    and densities (split-K and CTA-pair plans among them) in one pipelined
    call, each equal to the oracle; a second call reuses the workspace."""
    import bsp

    rng = np.random.default_rng(23)
    jobs, golds = [], []
    # N = 1024 and 8192 run as 2 and 4 column panels of one plan
    for M, K, N, R, C, p in [(4096, 4096, 1024, 32, 32, 0.5), (1024, 2048, 256, 64, 64, 0.2),
                             (2048, 1024, 512, 32, 32, 0.01), (512, 512, 96, 32, 64, 0.3),
                             (512, 1024, 8192, 64, 64, 0.2)]:
        rp, ci, vals = rand_bsr(rng, M, K, R, C, p, empty_rows=(1,))
        B = rand_dense(rng, K, N)
        jobs.append(dict(M=M, K=K, R=R, C=C, row_ptr=rp, col_idx=ci, values=vals, B=B, N=N))
        golds.append(oracle.spmm_bf16(rp, ci, vals, M, K, R, C, B, N))
    for _ in range(2):
        outs = bsp.spmm_host_batch(jobs, strategy=bsp.STRATEGIES[strategy])
        for k, (o, g) in enumerate(zip(outs, golds)):
            assert_bf16_close(o, g, what=f"batch job {k} {strategy}")
