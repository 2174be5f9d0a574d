"""SpGEMM host logic without a GPU: the planner's output pattern against the
oracle's symbolic product (bit-exact), and the planner's schedule executed by
a float64 emulator of the kernel (units, steps, zero boxes, epilogue tiles)
against the dense float64 product, so that every stored block product is
taken exactly once and every output tile is written exactly once."""
import glob
import os

import numpy as np
import pytest

import bsp
import oracle

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


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


def dense(rp, ci, vals, R, C, H, W):
    out = np.zeros((H, W))
    v = vals.reshape(-1, R, C)
    for i in range(rp.size - 1):
        for b in range(rp[i], rp[i + 1]):
            out[i * R:(i + 1) * R, ci[b] * C:(ci[b] + 1) * C] += v[b]
    return out


def emulate(plan, Ra, Ca, Cb, av, bv, nnzb_out):
    """Run the schedule the way the kernel does (float64): every step's TMA
    boxes fill the entry and segment slots (zero boxes for absent data), the
    MMA accumulates, the epilogue writes the tiles of existing blocks."""
    a2 = av.reshape(-1, Ca)
    b3 = bv.reshape(-1, Ca, Cb)
    nseg_max = plan["nseg_max"]
    out = np.full((nnzb_out, Ra, Cb), np.nan)
    written = np.zeros((nnzb_out, Ra, Cb), np.int32)
    steps = plan["step_table"]
    cta = plan["cta_begin"]
    assert cta[0] == 0 and cta[-1] == plan["units"] and np.all(np.diff(cta) >= 0)
    n_boxes = 0
    for u in plan["unit_table"]:
        sb, ns, n_ent, nseg = u[:4]
        seg_x, ent_r, out_blk = u[4:12], u[12:16], u[16:48].reshape(4, 8)
        assert ns >= 1 and 1 <= n_ent <= 4 and 1 <= nseg <= nseg_max
        D = np.zeros((128, 32 * nseg_max))
        for st in steps[sb:sb + ns]:
            meta = st[12:16].copy().view(np.uint8)
            a_meta, b_meta = meta[0:4], meta[4:12]
            A = np.full((128, Ca), np.nan)
            B = np.full((Ca, 32 * nseg_max), np.nan)
            cover_a = np.zeros(4, np.int32)
            cover_b = np.zeros(8, np.int32)
            for i in range(4):
                m = int(a_meta[i])
                if not m & 0x80:
                    continue
                n_boxes += 1
                e0, L = m & 7, 1 << ((m >> 3) & 3)
                y = st[i]
                assert e0 + L <= 4 and L <= 4
                cover_a[e0:e0 + L] += 1
                if y >= 0:
                    assert y + 32 * L <= a2.shape[0]
                    A[32 * e0:32 * (e0 + L)] = a2[y:y + 32 * L]
                else:
                    assert y == -32 * L
                    A[32 * e0:32 * (e0 + L)] = 0
            for i in range(8):
                m = int(b_meta[i])
                if not m & 0x80:
                    continue
                n_boxes += 1
                s0, L, t = m & 7, 1 << ((m >> 3) & 3), (m >> 5) & 3
                z = st[4 + i]
                assert s0 + L <= nseg
                cover_b[s0:s0 + L] += 1
                for q in range(L):
                    if z >= 0:
                        assert z + L <= b3.shape[0]
                        assert seg_x[s0 + q] == 32 * t
                        B[:, 32 * (s0 + q):32 * (s0 + q + 1)] = b3[z + q, :, 32 * t:32 * t + 32]
                    else:
                        assert z == -L
                        B[:, 32 * (s0 + q):32 * (s0 + q + 1)] = 0
            assert np.all(cover_a == 1), "every entry slot filled by exactly one box"
            assert np.all(cover_b[:nseg] == 1) and np.all(cover_b[nseg:] == 0)
            # rows of inactive entries / columns of unused segments stay out of the result
            A[np.isnan(A)] = 0
            B[:, 32 * nseg:] = 0
            D += A @ B
        for e in range(4):
            for s in range(8):
                blk = out_blk[e, s]
                if blk < 0:
                    continue
                assert e < n_ent and s < nseg
                out[blk, ent_r[e]:ent_r[e] + 32, seg_x[s]:seg_x[s] + 32] = D[32 * e:32 * e + 32, 32 * s:32 * s + 32]
                written[blk, ent_r[e]:ent_r[e] + 32, seg_x[s]:seg_x[s] + 32] += 1
    assert np.all(written == 1), "every output element written exactly once"
    assert n_boxes == plan["boxes"]
    return out


def check_case(rng, M, K, N, Ra, Ca, Cb, arp, aci, brp, bci, **opts):
    av = oracle.bf16_to_f32(oracle.f32_to_bf16(rng.uniform(-1, 1, aci.size * Ra * Ca).astype(np.float32)))
    bv = oracle.bf16_to_f32(oracle.f32_to_bf16(rng.uniform(-1, 1, bci.size * Ca * Cb).astype(np.float32)))
    plan = bsp.inspect_spgemm_plan(M, K, N, Ra, Ca, Cb, arp, aci, brp, bci, opts=bsp.make_opts(**opts))
    orp, oci = oracle.spgemm_pattern(arp, aci, brp, bci, N // Cb)
    assert np.array_equal(plan["out_row_ptr"], orp) and np.array_equal(plan["out_col_idx"], oci)
    pairs = sum(int(brp[aci[a] + 1] - brp[aci[a]]) for a in range(aci.size))
    assert plan["pairs"] == pairs and plan["out_nnzb"] == oci.size
    got = emulate(plan, Ra, Ca, Cb, av.astype(np.float64), bv.astype(np.float64), oci.size)
    full = dense(arp, aci, av, Ra, Ca, M, K) @ dense(brp, bci, bv, Ca, Cb, K, N)
    for i in range(orp.size - 1):
        for q in range(orp[i], orp[i + 1]):
            j = oci[q]
            np.testing.assert_allclose(got[q], full[i * Ra:(i + 1) * Ra, j * Cb:(j + 1) * Cb], rtol=1e-9, atol=1e-9)
    return plan


@pytest.mark.parametrize("Ra,Ca,Cb", [(32, 32, 32), (64, 32, 32), (128, 32, 32), (32, 64, 32),
                                      (32, 128, 32), (32, 32, 64), (32, 32, 128), (64, 64, 64),
                                      (128, 128, 128)])
def test_schedule_emulates_product(Ra, Ca, Cb):
    rng = np.random.default_rng(Ra * 3 + Ca * 5 + Cb * 7)
    nbr, nbk, nbc = 11, 9, 13
    arp, aci = rand_pattern(rng, nbr, nbk, 0.3, empty_rows=(2,))
    brp, bci = rand_pattern(rng, nbk, nbc, 0.3, empty_rows=(1,))
    plan = check_case(rng, nbr * Ra, nbk * Ca, nbc * Cb, Ra, Ca, Cb, arp, aci, brp, bci)
    assert plan["kc"] == (32 if Ca == 32 else 64)


@pytest.mark.parametrize("opts", [dict(n_tiles=1), dict(n_tiles=2), dict(steps_per_stage=1),
                                  dict(steps_per_stage=4), dict(no_load_balance=1),
                                  dict(no_load_balance=2), dict(max_ctas=3), dict(producers=1)])
def test_schedule_options(opts):
    rng = np.random.default_rng(11)
    arp, aci = rand_pattern(rng, 14, 10, 0.35)
    brp, bci = rand_pattern(rng, 10, 12, 0.35)
    plan = check_case(rng, 14 * 32, 10 * 32, 12 * 32, 32, 32, 32, arp, aci, brp, bci, **opts)
    if "n_tiles" in opts:
        assert plan["nseg_max"] == 4 * opts["n_tiles"]
    if "max_ctas" in opts:
        assert plan["ctas"] <= 3
    assert plan["stages"] % plan["producers"] == 0


@pytest.mark.parametrize("Ra,Cb", [(32, 32), (64, 64)])
def test_repeated_and_unsorted_columns(Ra, Cb):
    """Rows of A and of B holding the same column twice contribute every pair."""
    rng = np.random.default_rng(5)
    arp, aci = rand_pattern(rng, 9, 6, 0.4, repeats=2)
    brp, bci = rand_pattern(rng, 6, 7, 0.4, repeats=2)
    assert any(len(set(aci[arp[i]:arp[i + 1]])) < arp[i + 1] - arp[i] for i in range(9))
    check_case(rng, 9 * Ra, 6 * 32, 7 * Cb, Ra, 32, Cb, arp, aci, brp, bci)


def test_empty_product_and_empty_inputs():
    rng = np.random.default_rng(2)
    # A's columns never meet B's stored rows
    arp = np.array([0, 1, 2], np.int32)
    aci = np.array([0, 0], np.int32)
    brp = np.array([0, 0, 2], np.int32)
    bci = np.array([0, 1], np.int32)
    plan = check_case(rng, 64, 64, 64, 32, 32, 32, arp, aci, brp, bci)
    assert plan["out_nnzb"] == 0 and plan["units"] == 0 and plan["ctas"] == 0
    # A with no blocks at all
    plan = check_case(rng, 64, 64, 64, 32, 32, 32, np.zeros(3, np.int32), np.zeros(0, np.int32), brp, bci)
    assert plan["out_nnzb"] == 0


def test_reference_fill_patterns_schedule():
    """The reference's own generator patterns (committed fixtures)."""
    rng = np.random.default_rng(9)
    for f in sorted(glob.glob(os.path.join(GOLDEN, "spgemm_*.npz"))):
        z = np.load(f)
        Ra, Ca, Cb = int(z["Ra"]), int(z["Ca"]), int(z["Cb"])
        check_case(rng, int(z["Ha"]), int(z["Wa"]), int(z["Wb"]), Ra, Ca, Cb, z["a_indptr"],
                   z["a_indices"], z["b_indptr"], z["b_indices"])


def test_unit_shape_banded():
    """A banded product packs full units: 4 entries x 8 segments."""
    n = 64
    rows = [[c for c in range(max(0, i - 2), min(n, i + 3))] for i in range(n)]
    rp = np.concatenate([[0], np.cumsum([len(r) for r in rows])]).astype(np.int32)
    ci = np.array([c for r in rows for c in r], np.int32)
    plan = bsp.inspect_spgemm_plan(n * 32, n * 32, n * 32, 32, 32, 32, rp, ci, rp, ci,
                                   opts=bsp.make_opts(n_tiles=2))
    assert plan["nseg_max"] == 8
    u = plan["unit_table"]
    assert np.all(u[:, 2] == 4)
    # an interior group of 4 rows covers 12 output columns (one unit of 8 and
    # one of 4); the first and last groups cover 8 (one unit)
    assert plan["units"] == 2 * (n // 4) - 2
    # each unit's steps: k in the union of its rows' bands that reach its columns
    assert plan["steps"] <= plan["units"] * 8
    # consecutive stored blocks of a row of B merge: far fewer than 12 boxes a step
    assert plan["boxes"] < 7 * plan["steps"]


def test_bad_arguments():
    rp = np.array([0, 1], np.int32)
    ci = np.array([0], np.int32)
    with pytest.raises(bsp.BspError):
        bsp.inspect_spgemm_plan(32, 32, 32, 32, 48, 32, rp, ci, rp, ci)  # block size
    with pytest.raises(bsp.BspError):
        bsp.inspect_spgemm_plan(32, 32, 40, 32, 32, 32, rp, ci, rp, ci)  # N % Cb
    with pytest.raises(bsp.BspError):
        bsp.inspect_spgemm_plan(32, 32, 32, 32, 32, 32, rp, np.array([3], np.int32), rp, ci)


def test_unit_width_choice():
    """Sparse random products get 4-segment units (N = 128) when those move
    fewer operand bytes; wide bands keep 8 (N = 256)."""
    rng = np.random.default_rng(21)
    arp, aci = rand_pattern(rng, 256, 256, 0.03)
    brp, bci = rand_pattern(rng, 256, 256, 0.03)
    p = bsp.inspect_spgemm_plan(256 * 32, 256 * 32, 256 * 32, 32, 32, 32, arp, aci, brp, bci)
    assert p["nseg_max"] == 4
    n = 128
    rows = [list(range(max(0, i - 16), min(n, i + 17))) for i in range(n)]
    rp = np.concatenate([[0], np.cumsum([len(r) for r in rows])]).astype(np.int32)
    ci = np.array([c for r in rows for c in r], np.int32)
    p = bsp.inspect_spgemm_plan(n * 32, n * 32, n * 32, 32, 32, 32, rp, ci, rp, ci)
    assert p["nseg_max"] == 8


@pytest.mark.parametrize("Ra,Cb", [(32, 32), (64, 32), (32, 64)])
def test_plan_independent_of_planner_threads(monkeypatch, Ra, Cb):
    """The planner splits block-rows and row groups over host threads and
    appends the pieces in order: the output pattern, units, steps and CTA
    ranges are the same for any thread count."""
    rng = np.random.default_rng(31 + Ra + Cb)
    arp, aci = rand_pattern(rng, 96, 80, 0.06, empty_rows=(5, 6), repeats=2)
    brp, bci = rand_pattern(rng, 80, 90, 0.06, empty_rows=(3,), repeats=1)
    plans = []
    for threads in ("1", "3", "7"):
        monkeypatch.setenv("BSP_PLANNER_THREADS", threads)
        plans.append(bsp.inspect_spgemm_plan(96 * Ra, 80 * 32, 90 * Cb, Ra, 32, Cb, arp, aci, brp, bci))
    for p in plans[1:]:
        for key in ("out_row_ptr", "out_col_idx", "unit_table", "step_table", "cta_begin"):
            assert np.array_equal(p[key], plans[0][key]), key
        assert all(p[k] == plans[0][k] for k in bsp.SPGEMM_INFO_KEYS)
    monkeypatch.setenv("BSP_PLANNER_THREADS", "4")
    check_case(rng, 96 * Ra, 80 * 32, 90 * Cb, Ra, 32, Cb, arp, aci, brp, bci)
