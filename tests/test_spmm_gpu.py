"""SpMM parity on the GPU: libbsp (through the C ABI) vs the CPU oracle.

Cases mirror the reference's own SpMM registry (block_spmm/inc/test_suite.hpp:
single blocks, diagonal/row/column fills, nonsquare and tall/wide blocks, empty
rows, wide N, large R) at sizes the oracle finishes in seconds, plus
BASELINE config 1 in full.  Bar: max relative error <= 1e-2 against the
bf16 golden (oracle restatement of bsr_matrix::spmm_bfloat16) and a normwise
error <= 1e-5 of the f32 output against the float golden.
"""
import numpy as np
import pytest

import oracle
from helpers import TOL, assert_bf16_close, normwise, pcc, rand_bsr, rand_dense

pytestmark = pytest.mark.gpu


def _bsp():
    import bsp

    return bsp


# strategy names of the reference plus the two DDA kernels forced explicitly
# (plain "dda" picks between them by estimated cost)
VARIANTS = {"naive": ("naive", {}), "snf": ("snf", {}), "dda": ("dda", {}),
            "dda_1cta": ("dda", {"group_mma": 4}), "dda_pair": ("dda", {"group_mma": 5}),
            "dda_twin": ("dda", {"group_mma": 6}), "dda_wide": ("dda", {"group_mma": 4, "n_tiles": 4})}
# dda_wide only differs from dda_1cta when N is a multiple of 512 (its own test)
STRATS = [v for v in VARIANTS if v != "dda_wide"]


def _sv(bsp, name, **extra):
    """(strategy id, Opts) of a VARIANTS name, with extra option fields."""
    s, o = VARIANTS[name]
    return bsp.STRATEGIES[s], bsp.make_opts(**{**o, **extra})

# (M, K, N, R, C, density)
CASES = [
    (1024, 1024, 256, 32, 32, 0.10),
    (256, 256, 256, 64, 64, 0.5),
    (256, 256, 256, 64, 32, 0.4),       # test_2_blocks_nonsquare-like
    (256, 256, 256, 32, 64, 0.4),
    (512, 512, 128, 128, 32, 0.3),      # tall blocks
    (256, 512, 96, 32, 128, 0.3),       # wide blocks
    (512, 256, 384, 256, 64, 0.5),      # big block
    (1024, 512, 64, 512, 64, 0.5),      # R > 256: two 256-row slabs per block
    (1024, 256, 32, 1024, 64, 0.6),     # test_huge-like R = 1024, N = 32
    (4096, 256, 40, 32, 32, 0.2),       # many rows, N not a multiple of 32
    (128, 4096, 8, 32, 32, 0.5),        # long rows (K = 4096), N = 8
    (384, 384, 200, 96, 64, 0.4),       # R = 96 (three 32-row chunks), N % 128 != 0
]


def _run(bsp, M, K, N, R, C, rp, ci, vals, B, strategy, c_type=0, opts=None):
    import torch

    A = bsp.DeviceBSR.from_host(M, K, R, C, rp, ci, vals)
    Bd = bsp.to_device_bf16(B)
    sid, vopts = _sv(bsp, strategy)
    out = bsp.spmm(A, Bd, strategy=sid, c_type=c_type, opts=opts if opts is not None else vopts)
    if c_type == bsp.F32:
        return out.cpu().numpy()
    return bsp.to_host_bits(out)


@pytest.mark.parametrize("case", CASES, ids=[f"{c[0]}x{c[1]}x{c[2]}_R{c[3]}C{c[4]}" for c in CASES])
@pytest.mark.parametrize("strategy", STRATS)
def test_spmm_parity(case, strategy):
    bsp = _bsp()
    M, K, N, R, C, p = case
    rng = np.random.default_rng(abs(hash((case, 1))) % 2**32)
    rp, ci, vals = rand_bsr(rng, M, K, R, C, p, empty_rows=(0,) if M // R > 2 else ())
    B = rand_dense(rng, K, N)
    gold = oracle.spmm_bf16(rp, ci, vals, M, K, R, C, B, N)
    out = _run(bsp, M, K, N, R, C, rp, ci, vals, B, strategy)
    assert_bf16_close(out, gold, what=f"{case} {strategy}")
    assert pcc(oracle.bf16_to_f32(out), oracle.bf16_to_f32(gold)) >= 0.99


@pytest.mark.parametrize("strategy", STRATS)
def test_spmm_f32_output_vs_float_golden(strategy):
    bsp = _bsp()
    M, K, N, R, C = 512, 512, 256, 32, 32
    rng = np.random.default_rng(11)
    rp, ci, vals = rand_bsr(rng, M, K, R, C, 0.3, empty_rows=(3,))
    B = rand_dense(rng, K, N)
    gold = oracle.spmm_f32(rp, ci, oracle.bf16_to_f32(vals), M, K, R, C, oracle.bf16_to_f32(B), N)
    out = _run(bsp, M, K, N, R, C, rp, ci, vals, B, strategy, c_type=bsp.F32)
    assert normwise(out, gold) <= 1e-5
    e = np.abs(out - gold) / np.maximum(np.abs(gold), 1e-3 * np.abs(gold).max())
    assert e.max() <= 1e-4


def test_spmm_torch_fp32_reference():
    """Cross-check against a plain PyTorch fp32 dense product of the same op."""
    import torch

    bsp = _bsp()
    M, K, N, R, C = 1024, 1024, 512, 32, 32
    rng = np.random.default_rng(5)
    rp, ci, vals = rand_bsr(rng, M, K, R, C, 0.2)
    B = rand_dense(rng, K, N)
    dense = np.zeros((M, K), np.float32)
    v = oracle.bf16_to_f32(vals).reshape(-1, R, C)
    for i in range(M // R):
        for b in range(rp[i], rp[i + 1]):
            dense[i * R:(i + 1) * R, ci[b] * C:(ci[b] + 1) * C] = v[b]
    ref = (torch.from_numpy(dense).cuda() @ torch.from_numpy(oracle.bf16_to_f32(B)).cuda()).cpu().numpy()
    out = _run(bsp, M, K, N, R, C, rp, ci, vals, B, "dda", c_type=bsp.F32)
    assert normwise(out, ref) <= 1e-5


@pytest.mark.parametrize("strategy", STRATS)
def test_spmm_empty_matrix_writes_zeros(strategy):
    import torch

    bsp = _bsp()
    M, K, N, R, C = 256, 256, 128, 32, 32
    rp = np.zeros(M // R + 1, np.int32)
    ci = np.zeros(0, np.int32)
    A = bsp.DeviceBSR.from_host(M, K, R, C, rp, ci, np.zeros(0, np.uint16))
    B = bsp.to_device_bf16(rand_dense(np.random.default_rng(0), K, N))
    C_ = torch.full((M, N), 7.0, dtype=torch.bfloat16, device="cuda")
    sid, vopts = _sv(bsp, strategy)
    plan = bsp.SpmmPlan(bsp.device(), A, N, sid, opts=vopts)
    plan.execute(A, B, C_)
    bsp.device().synchronize()
    assert torch.count_nonzero(C_).item() == 0


@pytest.mark.parametrize("strategy", STRATS)
def test_spmm_overwrites_stale_output(strategy):
    """Every element of C is written, the rows of empty block-rows included."""
    import torch

    bsp = _bsp()
    M, K, N, R, C = 512, 256, 256, 32, 32
    rng = np.random.default_rng(3)
    rp, ci, vals = rand_bsr(rng, M, K, R, C, 0.2, empty_rows=(0, 1, 5, 15))
    B = rand_dense(rng, K, N)
    gold = oracle.spmm_bf16(rp, ci, vals, M, K, R, C, B, N)
    A = bsp.DeviceBSR.from_host(M, K, R, C, rp, ci, vals)
    C_ = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
    sid, vopts = _sv(bsp, strategy)
    plan = bsp.SpmmPlan(bsp.device(), A, N, sid, opts=vopts)
    plan.execute(A, bsp.to_device_bf16(B), C_)
    bsp.device().synchronize()
    assert_bf16_close(bsp.to_host_bits(C_), gold)


def test_spmm_duplicate_and_unsorted_columns():
    """A row may list columns out of order and even twice (both blocks count)."""
    bsp = _bsp()
    M, K, N, R, C = 128, 256, 128, 32, 32
    rp = np.array([0, 3, 3, 6, 7], np.int32)
    ci = np.array([5, 1, 5, 7, 0, 7, 2], np.int32)
    rng = np.random.default_rng(9)
    vals = oracle.f32_to_bf16(rng.uniform(-1, 1, ci.size * R * C).astype(np.float32))
    B = rand_dense(rng, K, N)
    gold = oracle.spmm_bf16(rp, ci, vals, M, K, R, C, B, N)
    for s in STRATS:
        out = _run(bsp, M, K, N, R, C, rp, ci, vals, B, s)
        assert_bf16_close(out, gold, what=s)


@pytest.mark.parametrize("opts", [dict(no_load_balance=1), dict(max_ctas=3), dict(group_rows=8, n_tiles=1),
                                  dict(group_rows=2, n_tiles=4), dict(n_tiles=3)])
def test_spmm_schedule_options(opts):
    bsp = _bsp()
    M, K, N, R, C = 1024, 512, 384, 32, 32
    rng = np.random.default_rng(21)
    rp, ci, vals = rand_bsr(rng, M, K, R, C, 0.15, empty_rows=(4, 5, 6))
    B = rand_dense(rng, K, N)
    gold = oracle.spmm_bf16(rp, ci, vals, M, K, R, C, B, N)
    strat = "dda" if "group_rows" in opts else "snf"
    out = _run(bsp, M, K, N, R, C, rp, ci, vals, B, strat, opts=bsp.make_opts(**opts))
    assert_bf16_close(out, gold, what=str(opts))


def test_spmm_strided_operands():
    import torch

    bsp = _bsp()
    M, K, N, R, C = 256, 256, 128, 32, 32
    rng = np.random.default_rng(4)
    rp, ci, vals = rand_bsr(rng, M, K, R, C, 0.4)
    B = rand_dense(rng, K, N)
    gold = oracle.spmm_bf16(rp, ci, vals, M, K, R, C, B, N)
    A = bsp.DeviceBSR.from_host(M, K, R, C, rp, ci, vals)
    Bbig = torch.zeros((K, N + 64), dtype=torch.bfloat16, device="cuda")
    Bbig[:, :N] = bsp.to_device_bf16(B)
    Cbig = torch.zeros((M, N + 32), dtype=torch.bfloat16, device="cuda")
    plan = bsp.SpmmPlan(bsp.device(), A, N, bsp.DDA)
    plan.execute(A, Bbig[:, :N], Cbig[:, :N])
    bsp.device().synchronize()
    assert_bf16_close(bsp.to_host_bits(Cbig[:, :N]), gold)
    assert torch.count_nonzero(Cbig[:, N:]).item() == 0


@pytest.mark.parametrize("strategy", STRATS)
def test_spmm_host_buffer_api(strategy):
    """The reference-semantics entry point: host arrays in, host C out."""
    bsp = _bsp()
    M, K, N, R, C = 1024, 1024, 256, 32, 32
    rng = np.random.default_rng(1234 + 0)
    rp, ci, vals = rand_bsr(rng, M, K, R, C, 0.10)
    B = rand_dense(rng, K, N)
    gold = oracle.spmm_bf16(rp, ci, vals, M, K, R, C, B, N)
    sid, vopts = _sv(bsp, strategy)
    out = bsp.spmm_host(M, K, R, C, rp, ci, vals, B, N, strategy=sid, opts=vopts)
    assert_bf16_close(out, gold)


def test_spmm_rejects_bad_arguments():
    bsp = _bsp()
    M, K, R, C = 256, 256, 32, 32
    rp = np.zeros(M // R + 1, np.int32)
    A = bsp.DeviceBSR.from_host(M, K, R, C, rp, np.zeros(0, np.int32), np.zeros(0, np.uint16))
    with pytest.raises(bsp.BspError):
        bsp.SpmmPlan(bsp.device(), A, 100, bsp.NAIVE)  # N % 8 != 0
    bad = bsp.DeviceBSR.from_host(M, K, 48, 32, np.zeros(M // 48 + 1, np.int32), np.zeros(0, np.int32), None)
    with pytest.raises(bsp.BspError):
        bsp.SpmmPlan(bsp.device(), bad, 128, bsp.NAIVE)  # R % 32 != 0
    rp2 = np.array([0, 1, 1, 1, 1, 1, 1, 1, 1], np.int32)
    A2 = bsp.DeviceBSR.from_host(M, K, R, C, rp2, np.array([99], np.int32), np.zeros(R * C, np.uint16))
    with pytest.raises(bsp.BspError):
        bsp.SpmmPlan(bsp.device(), A2, 128, bsp.NAIVE)  # column index out of range


@pytest.mark.parametrize("R,nonempty_rows,no_lb", [(64, 1, 0), (64, 1, 1), (256, 2, 1), (32, 3, 0)])
def test_pair_kernel_empty_first_units(R, nonempty_rows, no_lb):
    """CTA pairs whose lists start with (or are only) units without blocks:
    their stages are released by plain arrives, not by a 2-SM commit with no
    MMA before it; twenty launches each must finish and match the oracle."""
    import bsp
    import torch

    rng = np.random.default_rng(R + nonempty_rows)
    M = K = 2048
    N = 512
    nb = M // R
    occ = np.zeros((nb, K // R), bool)
    occ[:nonempty_rows] = rng.random((nonempty_rows, K // R)) < 0.8
    rp = np.concatenate([[0], np.cumsum(occ.sum(1))]).astype(np.int32)
    ci = np.nonzero(occ)[1].astype(np.int32)
    vals = rand_dense(rng, ci.size * R, R).ravel()
    B = rand_dense(rng, K, N)
    gold = oracle.spmm_bf16(rp, ci, vals, M, K, R, R, B, N)
    A = bsp.DeviceBSR.from_host(M, K, R, R, rp, ci, vals)
    Bd = bsp.to_device_bf16(B)
    C = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
    dev = bsp.device(0)
    plan = bsp.SpmmPlan(dev, A, N, bsp.DDA, bsp.BF16, bsp.make_opts(group_mma=5, no_load_balance=no_lb, timeout_ms=500))
    assert plan.info()["variant"] == 2
    for _ in range(20):
        C.fill_(float("nan"))
        plan.execute(A, Bd, C)
        dev.synchronize()
        assert_bf16_close(bsp.to_host_bits(C), gold, what=f"pair R={R}")
    plan.close()


def _skewed_rows(rng, nbr, nbc, heavy, heavy_len, light_len):
    rows = [sorted(rng.choice(nbc, heavy_len if i in heavy else light_len, replace=False)) for i in range(nbr)]
    rp = np.concatenate([[0], np.cumsum([len(r) for r in rows])]).astype(np.int32)
    return rp, np.concatenate(rows).astype(np.int32)


@pytest.mark.parametrize("variant,N", [("dda_1cta", 128), ("dda_1cta", 256), ("dda_pair", 256), ("dda", 200)])
@pytest.mark.parametrize("c_f32", [False, True])
def test_spmm_split_k_parity(variant, N, c_f32):
    """Block-rows far longer than the rest get split-K: parts of a unit over
    consecutive step ranges leave fp32 partial tiles in the plan's workspace
    and the last part to finish sums them and stores C.  The result matches
    the oracle, and a second launch of the same plan (counters reset by the
    merging parts) gives the same bits."""
    import torch

    bsp = _bsp()
    R = C = 32
    M, K = 4096, 8192
    rng = np.random.default_rng(N + 7 * c_f32)
    rp, ci = _skewed_rows(rng, M // R, K // C, heavy={3, 4, 5, 40, 41, 90}, heavy_len=230, light_len=5)
    vals = oracle.f32_to_bf16(rng.uniform(-1, 1, ci.size * R * C).astype(np.float32))
    B = rand_dense(rng, K, N)
    sid, opts = _sv(bsp, variant)
    plan_info = bsp.inspect_spmm_plan(M, K, R, C, rp, ci, N, sid, opts=opts)
    assert ((plan_info["unit_table"][:, 4] & 0xFF) > 1).any()       # split-K is in the plan
    A = bsp.DeviceBSR.from_host(M, K, R, C, rp, ci, vals)
    Bd = bsp.to_device_bf16(B)
    dev = bsp.device()
    ctype = bsp.F32 if c_f32 else bsp.BF16
    plan = bsp.SpmmPlan(dev, A, N, sid, ctype, opts)
    outs = []
    for _ in range(2):
        Cd = torch.full((M, N), float("nan"), dtype=torch.float32 if c_f32 else torch.bfloat16, device="cuda")
        plan.execute(A, Bd, Cd)
        dev.synchronize()
        outs.append(Cd.cpu().numpy() if c_f32 else bsp.to_host_bits(Cd))
    plan.close()
    assert np.array_equal(outs[0], outs[1])
    if c_f32:
        gold = oracle.spmm_f32(rp, ci, oracle.bf16_to_f32(vals), M, K, R, C, oracle.bf16_to_f32(B), N)
        assert normwise(outs[0], gold) <= 1e-5
    else:
        gold = oracle.spmm_bf16(rp, ci, vals, M, K, R, C, B, N)
        assert_bf16_close(outs[0], gold, what=f"split-K {variant} N={N}")


@pytest.mark.parametrize("variant", ["dda_1cta", "dda_pair"])
def test_spmm_large_b_tile_order_parity(variant):
    """B of 128 MiB (more than fits in L2 beside A): the plan deals its units
    tile by tile (and may cut long ones); the result matches the oracle."""
    bsp = _bsp()
    M, K, N, R, C = 1024, 32768, 2048, 32, 32
    rng = np.random.default_rng(41)
    rp, ci, vals = rand_bsr(rng, M, K, R, C, 0.01)
    B = rand_dense(rng, K, N)
    gold = oracle.spmm_bf16(rp, ci, vals, M, K, R, C, B, N)
    out = _run(bsp, M, K, N, R, C, rp, ci, vals, B, variant)
    assert_bf16_close(out, gold, what=f"large B {variant}")


def _power_law_rows(rng, nbr, nbc, density, s=1.1):
    w = np.arange(1, nbr + 1, dtype=np.float64) ** -s
    counts = np.minimum(nbc, np.maximum(1, np.round(w * density * nbr * nbc / w.sum()))).astype(int)
    counts = counts[rng.permutation(nbr)]
    rows = [np.sort(rng.choice(nbc, size=c, replace=False)) for c in counts]
    rp = np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)
    return rp, np.concatenate(rows).astype(np.int32)


@pytest.mark.parametrize("R,N,c_f32", [(64, 512, False), (32, 296, False), (32, 256, True), (64, 128, True)])
def test_spmm_length_ordered_stacking_parity(R, N, c_f32):
    """Power-law block-row lengths: the row-stacked kernel stacks rows longest
    first (the plan's entry order maps stack entries to block-rows and the
    epilogue writes each entry's rows where they belong).  All of C matches
    the oracle, empty rows included, and a relaunch gives the same bits."""
    import torch

    bsp = _bsp()
    M = K = 8192
    rng = np.random.default_rng(R * 3 + N + c_f32)
    rp, ci = _power_law_rows(rng, M // R, K // R, 0.02)
    vals = oracle.f32_to_bf16(rng.uniform(-1, 1, ci.size * R * R).astype(np.float32))
    B = rand_dense(rng, K, N)
    sid, opts = _sv(bsp, "dda_1cta")
    info = bsp.inspect_spmm_plan(M, K, R, R, rp, ci, N, sid, opts=opts)
    assert info["entry_rows"] is not None
    A = bsp.DeviceBSR.from_host(M, K, R, R, rp, ci, vals)
    Bd = bsp.to_device_bf16(B)
    dev = bsp.device()
    plan = bsp.SpmmPlan(dev, A, N, sid, bsp.F32 if c_f32 else bsp.BF16, opts)
    outs = []
    for _ in range(2):
        Cd = torch.full((M, N), float("nan"), dtype=torch.float32 if c_f32 else torch.bfloat16, device="cuda")
        plan.execute(A, Bd, Cd)
        dev.synchronize()
        outs.append(Cd.cpu().numpy() if c_f32 else bsp.to_host_bits(Cd))
    plan.close()
    assert np.array_equal(outs[0], outs[1])
    if c_f32:
        gold = oracle.spmm_f32(rp, ci, oracle.bf16_to_f32(vals), M, K, R, R, oracle.bf16_to_f32(B), N)
        assert normwise(outs[0], gold) <= 1e-5
    else:
        gold = oracle.spmm_bf16(rp, ci, vals, M, K, R, R, B, N)
        assert_bf16_close(outs[0], gold, what=f"length-ordered stacking R={R} N={N}")


@pytest.mark.parametrize("R,N,c_f32,skew", [(64, 512, False, False), (32, 1024, False, False), (64, 1024, True, False),
                                          (32, 512, False, True), (64, 512, True, True)])
def test_spmm_wide_units_parity(R, N, c_f32, skew):
    """Wide units (opts.n_tiles = 4): 512 output columns in one TMEM
    accumulator, two N = 256 MMAs per k-step, 32-deep k-chunks.  With skewed
    rows the plan also cuts long units (split-K partials of 512 columns).
    All of C matches the oracle and a relaunch gives the same bits."""
    import torch

    bsp = _bsp()
    M, K = 2048, 8192
    rng = np.random.default_rng(R + N + 5 * c_f32 + 11 * skew)
    if skew:
        rp, ci = _skewed_rows(rng, M // R, K // R, heavy={1, 2, 9, 30}, heavy_len=100, light_len=3)
        vals = oracle.f32_to_bf16(rng.uniform(-1, 1, ci.size * R * R).astype(np.float32))
    else:
        rp, ci, vals = rand_bsr(rng, M, K, R, R, 0.05)
    B = rand_dense(rng, K, N)
    sid, opts = _sv(bsp, "dda_wide")
    info = bsp.inspect_spmm_plan(M, K, R, R, rp, ci, N, sid, opts=opts)
    assert info["n_tiles"] == 4 and info["tmem_cols"] == 512
    if skew:
        assert ((info["unit_table"][:, 4] & 0xFF) > 1).any()
    A = bsp.DeviceBSR.from_host(M, K, R, R, rp, ci, vals)
    Bd = bsp.to_device_bf16(B)
    dev = bsp.device()
    plan = bsp.SpmmPlan(dev, A, N, sid, bsp.F32 if c_f32 else bsp.BF16, opts)
    outs = []
    for _ in range(2):
        Cd = torch.full((M, N), float("nan"), dtype=torch.float32 if c_f32 else torch.bfloat16, device="cuda")
        plan.execute(A, Bd, Cd)
        dev.synchronize()
        outs.append(Cd.cpu().numpy() if c_f32 else bsp.to_host_bits(Cd))
    plan.close()
    assert np.array_equal(outs[0], outs[1])
    if c_f32:
        gold = oracle.spmm_f32(rp, ci, oracle.bf16_to_f32(vals), M, K, R, R, oracle.bf16_to_f32(B), N)
        assert normwise(outs[0], gold) <= 1e-5
    else:
        gold = oracle.spmm_bf16(rp, ci, vals, M, K, R, R, B, N)
        assert_bf16_close(outs[0], gold, what=f"wide units R={R} N={N} skew={skew}")
