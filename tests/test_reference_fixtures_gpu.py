"""GPU parity on the reference's own structural fixtures.

The patterns were read from the reference's headers by
tests/golden/make_golden.py and stored with goldens that the reference's CPU
golden (oracle/_ref) computed at sampled positions:

* all 36 frozen random patterns of block_spmm/inc/profiling_suite.hpp
  (make_frozen_case, 69-91: block values 1.0, dense operand the RAND kind after
  srand(42)), run through the reference's three strategies;
* test_random_hang / test_random_hang_v2 (block_spmm/inc/test_suite.hpp:
  584-646), run through every SpMM kernel variant;
* the SDDMM deadlock repro test_deadlock_sweepK_0
  (block_sddmm/inc/test_suite.hpp:112-171), run through Naive, SnF and CDA.

The inputs are regenerated from the stored seed with oracle.rand_fill (the C
library rand() draws of the reference generators), checked against the stored
first values.  Each output is compared with the stored reference golden at
the sampled positions, with the oracle restatement on whole block-rows or the
whole output, and (frozen patterns) by the product with a random vector,
C v = A (B v), over the whole output.
"""
import os

import numpy as np
import pytest

import oracle
from helpers import TOL, assert_bf16_close

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
_FROZEN = np.load(os.path.join(GOLDEN, "spmm_frozen_profiling_suite.npz"))
FROZEN_TAGS = sorted({k.split("__")[0] for k in _FROZEN.files if "__" in k})
ONE_BF16 = 0x3F80

# kernels of the SpMM path: the reference's three strategies, plus the two
# DDA kernels forced explicitly ("dda" picks between them by estimated cost)
SPMM_VARIANTS = {"naive": ("naive", {}), "snf": ("snf", {}), "dda": ("dda", {}),
                 "dda_1cta": ("dda", {"group_mma": 4}), "dda_pair": ("dda", {"group_mma": 5}),
                 "dda_twin": ("dda", {"group_mma": 6})}


def _spmm_dev(bsp, A, Bd, name):
    s, o = SPMM_VARIANTS[name]
    return bsp.spmm(A, Bd, strategy=bsp.STRATEGIES[s], opts=bsp.make_opts(**o))


def _rand_dense(K, N, seed, b_head=None):
    _, s = oracle.rand_fill(seed, 0, K * N)
    B = oracle.f32_to_bf16(s).reshape(K, N)
    if b_head is not None:
        assert np.array_equal(B.reshape(-1)[:b_head.size], b_head), "generator drifted from the fixture"
    return B


def _rows_oracle(ip, ix, vals, K, R, C, B, blocks, cols):
    """Oracle rows of the block-rows `blocks` at the columns `cols`: the
    product of the sub-matrix of those block-rows with B[:, cols]."""
    sub_ip, sub_ix, sub_v = [0], [], []
    vv = vals.reshape(-1, R * C)
    for b in blocks:
        sub_ix.append(ix[ip[b]:ip[b + 1]])
        sub_v.append(vv[ip[b]:ip[b + 1]])
        sub_ip.append(sub_ip[-1] + int(ip[b + 1] - ip[b]))
    six = np.concatenate(sub_ix).astype(np.int32)
    sv = np.concatenate(sub_v).reshape(-1)
    Bs = np.ascontiguousarray(B[:, cols])
    return oracle.spmm_bf16(np.array(sub_ip, np.int32), six, sv, len(blocks) * R, K, R, C, Bs, cols.size)


def _product_check(Cd, ip, ix, vals, R, C, Bd, seed):
    """||C v - A (B v)|| / || |C| |v| || for a random sign vector v, with B v
    and C v on the GPU in fp32 and A (B v) on the host in fp64.  The
    denominator (row sums of |C|) has no cancellation, so the bound holds for
    rows whose signed sum nearly cancels; rounding C to bf16 alone gives at
    most 2^-9 here."""
    import torch

    N = Bd.shape[1]
    v = torch.from_numpy(np.random.default_rng(seed).choice([-1.0, 1.0], N).astype(np.float32)).cuda()
    cv = (Cd.float() @ v).double().cpu().numpy()
    scale = Cd.float().abs().sum(1).double().cpu().numpy()
    w = (Bd.float() @ v).double().cpu().numpy()
    y = np.zeros(Cd.shape[0], np.float64)
    blocks = oracle.bf16_to_f32(vals).reshape(-1, R, C).astype(np.float64)
    rows = np.repeat(np.arange(ip.size - 1), np.diff(ip))
    if ix.size:
        contrib = np.einsum("brc,bc->br", blocks, w.reshape(-1, C)[ix])
        np.add.at(y.reshape(-1, R), rows, contrib)
    den = np.linalg.norm(scale)
    return 0.0 if den == 0 else float(np.linalg.norm(cv - y) / den)


@pytest.mark.parametrize("tag", FROZEN_TAGS)
def test_frozen_profiling_pattern(tag):
    import bsp

    z = _FROZEN
    M, N, K, R, C, _ = (int(x) for x in z[f"{tag}__shape"])
    ip, ix = z[f"{tag}__indptr"], z[f"{tag}__indices"]
    rows, cols, gold = z[f"{tag}__rows"], z[f"{tag}__cols"], z[f"{tag}__out"]
    B = _rand_dense(K, N, int(z["b_seed"]), z[f"{tag}__b_head"])
    vals = np.full(ix.size * R * C, ONE_BF16, np.uint16)
    A = bsp.DeviceBSR.from_host(M, K, R, C, ip, ix, vals)
    Bd = bsp.to_device_bf16(B)
    flops = 2.0 * ix.size * R * C * N
    full = oracle.spmm_bf16(ip, ix, vals, M, K, R, C, B, N) if flops <= 2.5e10 else None
    part = None
    if full is None:
        # whole sampled block-rows against the oracle on a 512-column window
        blocks = np.unique(rows // R)
        win = np.concatenate([np.arange(256), np.arange(N - 256, N)]) if N > 512 else np.arange(N)
        part = (blocks, win, _rows_oracle(ip, ix, vals, K, R, C, B, blocks, win))
    for name in ("dda", "naive", "snf"):
        Cd = _spmm_dev(bsp, A, Bd, name)
        out = bsp.to_host_bits(Cd)
        what = f"{tag} {name}"
        assert_bf16_close(out[np.ix_(rows, cols)], gold, what=what + " (reference golden)")
        if full is not None:
            assert_bf16_close(out, full, what=what + " (oracle)")
        else:
            blocks, win, g = part
            er = (blocks[:, None] * R + np.arange(R)[None, :]).reshape(-1)
            assert_bf16_close(out[np.ix_(er, win)], g, what=what + " (oracle, sampled block-rows)")
        assert _product_check(Cd, ip, ix, vals, R, C, Bd, seed=len(tag)) <= 1e-2, what


@pytest.mark.parametrize("name", ["spmm_test_random_hang", "spmm_test_random_hang_v2"])
@pytest.mark.parametrize("variant", list(SPMM_VARIANTS))
def test_random_hang_patterns(name, variant):
    import bsp

    z = np.load(os.path.join(GOLDEN, name + ".npz"))
    M, K, R, C, N = (int(z[k]) for k in ("H", "W", "R", "C", "N"))
    ip, ix = z["indptr"], z["indices"]
    u, s = oracle.rand_fill(int(z["seed"]), ix.size * R * C, K * N)
    vals = oracle.f32_to_bf16(u)
    B = oracle.f32_to_bf16(s).reshape(K, N)
    assert np.array_equal(B.reshape(-1)[:256], z["b_head"])
    A = bsp.DeviceBSR.from_host(M, K, R, C, ip, ix, vals)
    Bd = bsp.to_device_bf16(B)
    dev = bsp.device()
    out = None
    for _ in range(3):  # relaunches of the pattern the reference hung on
        out = bsp.to_host_bits(_spmm_dev(bsp, A, Bd, variant))
        dev.synchronize()
    assert_bf16_close(out[np.ix_(z["rows"], z["cols"])], z["out"], what=f"{name} {variant} (reference golden)")
    assert_bf16_close(out, oracle.spmm_bf16(ip, ix, vals, M, K, R, C, B, N), what=f"{name} {variant} (oracle)")


@pytest.mark.parametrize("strategy", ["naive", "snf", "dda"])
def test_sddmm_deadlock_pattern(strategy):
    import bsp

    z = np.load(os.path.join(GOLDEN, "sddmm_deadlock_sweepK_0.npz"))
    M, N, R, C, K = (int(z[k]) for k in ("H", "W", "R", "C", "K"))
    ip, ix = z["indptr"], z["indices"]
    nb = ix.size
    _, s = oracle.rand_fill(int(z["seed"]), 0, nb * R * C + M * K + K * N)
    mask = oracle.f32_to_bf16(s[:nb * R * C] * np.float32(2.0 ** int(z["mask_scale_log2"])))
    A = oracle.f32_to_bf16(s[nb * R * C:nb * R * C + M * K]).reshape(M, K)
    B = oracle.f32_to_bf16(s[nb * R * C + M * K:]).reshape(K, N)
    assert np.array_equal(A.reshape(-1)[:256], z["a_head"])
    out = bsp.sddmm_host(M, N, R, C, ip, ix, mask, A, B, K, strategy=bsp.STRATEGIES[strategy])
    ob = out.reshape(nb, R, C)
    got = ob[z["blocks"]][:, z["rows"]][:, :, z["cols"]]
    assert_bf16_close(got, z["out"], tol=TOL, what=f"deadlock {strategy} (reference golden)")
    gold = oracle.sddmm_bf16(ip, ix, mask, M, N, R, C, A, B, K)
    assert_bf16_close(out, gold, tol=TOL, what=f"deadlock {strategy} (oracle)")
