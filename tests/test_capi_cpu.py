"""CPU-side checks of the C ABI: every declared symbol is exported, the
host-only helpers behave, the planners' schedules cover the work exactly once,
and device calls fail cleanly without a GPU."""
import ctypes
import os
import re

import numpy as np
import pytest

import bsp
import oracle

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    names = set()
    for h in ("bsp.h", "bsp_testing.h"):
        src = open(os.path.join(ROOT, "include", h)).read()
        names |= set(re.findall(r"^\s*(?:bsp_status|int|const char\*)\s+(bsp_\w+)\(", src, re.M))
    return names


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(bsp.LIB_PATH)
    declared = _declared()
    assert len(declared) >= 25
    for name in sorted(declared):
        assert hasattr(lib, name), name
    assert set(bsp.EXPORTS) <= declared


def test_status_strings():
    L = bsp.lib()
    assert L.bsp_status_string(0) == b"ok"
    assert b"timed out" in L.bsp_status_string(4)


def test_device_open_fails_cleanly_without_gpu():
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(bsp.BspError):
        bsp.Device(0)


@pytest.mark.parametrize("n,parts", [(10, 4), (11, 4), (13, 4), (20, 4), (3, 8), (100, 7), (1, 1), (0, 3), (1000, 148)])
def test_serpentine_matches_oracle(n, parts):
    o1, s1 = bsp.serpentine_assign(n, parts)
    if n:
        o2, s2 = oracle.serpentine(n, parts)
        assert np.array_equal(o1, o2) and np.array_equal(s1, s2)


def _min_heaviest_range(w, parts):
    """Brute force: the least possible weight of the heaviest of `parts`
    contiguous ranges of w (dynamic programming over cut points)."""
    n = len(w)
    pre = np.concatenate([[0], np.cumsum(w)])
    INF = float("inf")
    best = [[INF] * (n + 1) for _ in range(parts + 1)]
    best[0][0] = 0
    for k in range(1, parts + 1):
        for j in range(n + 1):
            best[k][j] = min(max(best[k - 1][i], pre[j] - pre[i]) for i in range(j + 1))
    return best[parts][n]


def test_partition_rows_minimises_the_heaviest_range():
    """Power-law rows next to the cuts: the ranges reach the least possible
    heaviest range (blocks + one per row), and no range is over it."""
    rng = np.random.default_rng(5)
    for _ in range(40):
        nbr = int(rng.integers(1, 40))
        cnt = (rng.zipf(1.3, nbr).clip(0, 400) * rng.integers(0, 2, nbr)).astype(np.int64)
        rp = np.concatenate([[0], np.cumsum(cnt)]).astype(np.int32)
        for parts in (1, 2, 3, 5, 8):
            b = bsp.partition_rows(rp, parts)
            assert b[0] == 0 and b[-1] == nbr and np.all(np.diff(b) >= 0)
            w = [int(rp[b[i + 1]] - rp[b[i]] + (b[i + 1] - b[i])) for i in range(parts)]
            assert max(w) == _min_heaviest_range(cnt + 1, parts), (cnt.tolist(), parts, w)


def test_partition_rows_properties():
    rng = np.random.default_rng(0)
    for _ in range(50):
        nbr = int(rng.integers(1, 300))
        cnt = rng.zipf(1.5, nbr).clip(0, 500) * rng.integers(0, 2, nbr)
        rp = np.concatenate([[0], np.cumsum(cnt)]).astype(np.int32)
        for parts in (1, 2, 3, 8):
            b = bsp.partition_rows(rp, parts)
            assert b[0] == 0 and b[-1] == nbr and np.all(np.diff(b) >= 0)
            w = np.array([rp[b[i + 1]] - rp[b[i]] + (b[i + 1] - b[i]) for i in range(parts)])
            total = rp[-1] + nbr
            heaviest = max((cnt + 1).max(), 1)
            assert w.max() <= total / parts + heaviest  # within one row of the ideal split
