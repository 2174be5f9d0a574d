"""GPU outputs against the fixtures made by the reference's own golden
(tests/golden/*.npz): known-answer cases, reference fill patterns, BASELINE
config 1 and the SDDMM registry shapes, through every strategy."""
import glob
import os

import numpy as np
import pytest

import oracle
from helpers import assert_bf16_close, normwise

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
# SpMM and SDDMM fixtures that store their inputs (the SpGEMM ones are checked
# by test_spgemm_gpu.py, the seeded structural ones by
# test_reference_fixtures_gpu.py)
SEEDED = ("spmm_frozen_profiling_suite", "spmm_test_random_hang", "spmm_test_random_hang_v2",
          "sddmm_deadlock_sweepK_0")
FIXTURES = sorted(f for f in glob.glob(os.path.join(GOLDEN, "*.npz"))
                  if os.path.basename(f).startswith(("spmm_", "sddmm_"))
                  and os.path.basename(f)[:-4] not in SEEDED)


@pytest.mark.parametrize("path", FIXTURES, ids=[os.path.basename(f)[:-4] for f in FIXTURES])
@pytest.mark.parametrize("strategy", ["naive", "snf", "dda"])
def test_gpu_matches_reference_fixture(path, strategy):
    import bsp

    z = np.load(path)
    H, W, R, C = (int(z[k]) for k in ("H", "W", "R", "C"))
    if str(z["kind"]) == "spmm":
        N = int(z["N"])
        out = bsp.spmm_host(H, W, R, C, z["indptr"], z["indices"], z["values"], z["B"], N,
                            strategy=bsp.STRATEGIES[strategy])
        assert_bf16_close(out, z["out"], what=os.path.basename(path))
        # fp32 output against the float golden
        A = bsp.DeviceBSR.from_host(H, W, R, C, z["indptr"], z["indices"], z["values"])
        f = bsp.spmm(A, bsp.to_device_bf16(z["B"]), strategy=bsp.STRATEGIES[strategy], c_type=bsp.F32)
        assert normwise(f.cpu().numpy(), z["out_f32"]) <= 1e-5
    else:
        # Naive, SnF (the reference's unfinished store-and-forward SDDMM,
        # completed here) and CDA (DDA)
        K = int(z["K"])
        out = bsp.sddmm_host(H, W, R, C, z["indptr"], z["indices"], z["mask"], z["A"], z["B"], K,
                             strategy=bsp.STRATEGIES[strategy])
        assert_bf16_close(out, z["out"], what=os.path.basename(path))
