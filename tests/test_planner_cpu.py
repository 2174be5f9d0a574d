"""Planner invariants, checked on the CPU through the host-only inspect hook:
every output tile is produced by exactly one work unit, every block is
multiplied exactly once per tile, CTA lists partition the units, and the
row-stacked kernel's precomputed stage list (TMA coordinates, zero masks,
unit flags) is consistent with the schedule."""
import numpy as np
import pytest

import bsp
from helpers import rand_bsr

# DDA picks the single-CTA row-stacked kernel (variant 1) or the CTA-pair
# kernel (variant 2) by estimated cost; group_mma=4 / 5 force one of them.
STRATS = [("naive", {}), ("snf", {}), ("dda", dict(group_mma=4)), ("dda", dict(group_mma=4, steps_per_stage=1)),
          ("dda", dict(group_mma=2)), ("dda", dict(group_mma=3)), ("snf", dict(no_load_balance=1)),
          ("dda", dict(group_mma=4, n_tiles=4)),
          ("dda", dict(group_mma=4, no_load_balance=1, producers=2))]

SHAPES = [(1024, 1024, 256, 32, 32, 0.1), (512, 768, 200, 32, 32, 0.3), (512, 512, 384, 64, 64, 0.4),
          (768, 512, 128, 96, 32, 0.5), (1024, 512, 64, 512, 64, 0.5), (256, 256, 8, 32, 32, 0.0),
          (4096, 4096, 4096, 32, 32, 0.05)]


def _row_blocks(rp, i):
    return list(range(int(rp[i]), int(rp[i + 1])))


@pytest.mark.parametrize("shape", SHAPES, ids=[f"{s[0]}x{s[1]}x{s[2]}R{s[3]}C{s[4]}p{s[5]}" for s in SHAPES])
@pytest.mark.parametrize("strategy,opts", STRATS, ids=[f"{s}{o}" for s, o in STRATS])
def test_spmm_schedule_covers_work_exactly_once(shape, strategy, opts):
    M, K, N, R, C, p = shape
    rng = np.random.default_rng(int(M + K + N + R + 1000 * p))
    rp, ci, _ = rand_bsr(rng, M, K, R, C, p)
    plan = bsp.inspect_spmm_plan(M, K, R, C, rp, ci, N, bsp.STRATEGIES[strategy],
                                 opts=bsp.make_opts(**opts))
    _check_spmm_schedule(plan, rp, ci, M, N, R, C)


def _power_law_rows(rng, nbr, nbc, density, s=1.1):
    """Block-row lengths following Zipf's law over ranks (rows shuffled),
    columns uniform: the shape of config 5."""
    w = np.arange(1, nbr + 1, dtype=np.float64) ** -s
    counts = np.minimum(nbc, np.maximum(1, np.round(w * density * nbr * nbc / w.sum()))).astype(int)
    counts = counts[rng.permutation(nbr)]
    rp = np.zeros(nbr + 1, np.int32)
    rp[1:] = np.cumsum(counts)
    ci = np.concatenate([np.sort(rng.choice(nbc, size=c, replace=False)) for c in counts]).astype(np.int32)
    return rp, ci


@pytest.mark.parametrize("R,N", [(64, 512), (32, 296), (32, 128)])
def test_power_law_rows_stack_by_length(R, N):
    """Rows of very different lengths are stacked longest first (fewer
    union steps); the schedule still covers every block once per tile."""
    M = K = 8192
    rng = np.random.default_rng(R + N)
    rp, ci = _power_law_rows(rng, M // R, K // R, 0.02)
    plan = bsp.inspect_spmm_plan(M, K, R, R, rp, ci, N, bsp.DDA, opts=bsp.make_opts(group_mma=4))
    er = plan["entry_rows"]
    assert plan["variant"] == 1 and er is not None
    assert sorted(er.tolist()) == list(range(M // R))
    lens = np.diff(rp)[er]
    assert np.all(lens[:-1] >= lens[1:])
    _check_spmm_schedule(plan, rp, ci, M, N, R, R)
    # consecutive stacking of the same pattern needs more steps
    flat = bsp.inspect_spmm_plan(M, K, R, R, rp, ci, N, bsp.DDA, opts=bsp.make_opts(group_mma=4, no_load_balance=1))
    assert flat["entry_rows"] is None and flat["steps"] > plan["steps"]


def _check_spmm_schedule(plan, rp, ci, M, N, R, C):
    units, cta, steps = plan["unit_table"], plan["cta_begin"], plan["step_table"]
    assert cta[0] == 0 and cta[-1] == len(units) and np.all(np.diff(cta) >= 0)
    assert plan["ctas"] <= 148 and plan["stages"] >= 2
    G = plan["group_rows"]
    nbr = M // R
    if plan["variant"] == 1:
        Rs = plan["slab"]
        slabs = R // Rs
        assert G * Rs == 128
        tile_n = 128 * plan["n_tiles"]          # 256, or 128 when N <= 128, or 512 (wide units)
        wide = plan["tmem_cols"] == 512 and tile_n == 512
        assert tile_n == (512 if wide else 128 if N <= 128 else 256)
        assert not wide or (N % 512 == 0 and plan["kc"] == 32 and plan["nsub"] == 1)
        # units, or split-K parts of units: part (nt >> 8) of nt & 0xFF, slot r_off + part
        tiles, slots = {}, set()
        for u in units:
            row0, nent, r_off, n0, nt, sb, se, mask = (int(x) for x in u)
            assert n0 % tile_n == 0
            n_parts, part = nt & 0xFF, (nt >> 8) & 0xFF
            assert 1 <= n_parts <= 16 and part < n_parts
            if n_parts > 1:
                assert r_off + part not in slots and se - sb >= 1
                slots.add(r_off + part)
            else:
                assert r_off == 0
            tiles.setdefault((row0, n0), []).append((part, n_parts, r_off, sb, se, nent, mask))
        covered = {}
        for (row0, n0), parts in tiles.items():
            parts.sort()
            n_parts = parts[0][1]
            assert [q[0] for q in parts] == list(range(n_parts))
            assert all(q[1] == n_parts and q[2] == parts[0][2] and q[5:] == parts[0][5:] for q in parts)
            assert all(a[4] == b[3] for a, b in zip(parts, parts[1:]))   # consecutive step ranges
            sb, se, nent, mask = parts[0][3], parts[-1][4], parts[0][5], parts[0][6]
            blocks = {g: [] for g in range(G)}
            for s in range(sb, se):
                for g in range(G):
                    b = steps[s, 1 + g]
                    if b >= 0:
                        blocks[g].append(int(b))
                        assert ci[b] == steps[s, 0]
            er = plan["entry_rows"]
            for g in range(nent):
                e = row0 + g if er is None else int(er[row0 + g])
                covered[(e, n0)] = covered.get((e, n0), 0) + 1
                assert sorted(blocks[g]) == _row_blocks(rp, e // slabs)
                assert bool((mask >> g) & 1) == (rp[e // slabs + 1] > rp[e // slabs])
        assert len(covered) == nbr * slabs * ((N + tile_n - 1) // tile_n)
        assert all(v == 1 for v in covered.values())
        _check_stage_list(plan, rp, ci, R, C, Rs, slabs, G)
    else:
        Rs = plan["slab"]
        covered = {}
        for u in units:
            row0, nrows, r_off, n0, nt, sb, se, mask = (int(x) for x in u)
            blocks = {g: [] for g in range(G)}
            for s in range(sb, se):
                for g in range(G):
                    b = steps[s, 1 + g]
                    if b >= 0:
                        blocks[g].append(int(b))
                        assert ci[b] == steps[s, 0]
            for g in range(nrows):
                assert sorted(blocks[g]) == _row_blocks(rp, row0 + g)
                for t in range(nt):
                    key = (row0 + g, r_off, n0 + 128 * t)
                    covered[key] = covered.get(key, 0) + 1
        assert len(covered) == nbr * (R // Rs) * ((N + 127) // 128)
        assert all(v == 1 for v in covered.values())


def _check_stage_list(plan, rp, ci, R, C, Rs, slabs, G):
    """Replay each CTA's stage list against the units it runs."""
    units, cta, st, cst = plan["unit_table"], plan["cta_begin"], plan["stage_table"], plan["cta_stage_begin"]
    S, kc = plan["stages"], plan["kc"]
    nkc = C // kc
    FIRST, LAST, EMPTY, TWO = 1 << 24, 1 << 25, 1 << 26, 1 << 27
    for c in range(plan["ctas"]):
        rows = st[cst[c]:cst[c + 1]]
        state = np.full((S, 2), (1 << G) - 1, dtype=np.int64)  # slot contents unknown at start
        k = 0
        for ui in range(cta[c], cta[c + 1]):
            row0, nent, _, n0, _, sb, se, _ = (int(x) for x in units[ui])
            items = [(j, kci) for j in range(sb, se) for kci in range(nkc)]
            if not items:
                assert rows[k, 0] & (FIRST | LAST | EMPTY) == FIRST | LAST | EMPTY
                k += 1
                continue
            i = 0
            first = True
            while i < len(items):
                f = int(rows[k, 0])
                nsub = 2 if f & TWO else 1
                assert bool(f & FIRST) == first and not f & EMPTY
                first = False
                np_total = 0
                for q in range(nsub):
                    j, kci = items[i + q]
                    present = (f >> (4 * q)) & 0xF
                    zero = (f >> (8 + 4 * q)) & 0xF
                    for g in range(G):
                        b = plan["step_table"][j, 1 + g]
                        has = g < nent and b >= 0
                        assert bool((present >> g) & 1) == has
                        if has:
                            np_total += 1
                            assert rows[k, 5 + 4 * q + g] == b * R + ((row0 + g) % slabs) * Rs
                            assert plan["step_table"][j, 0] * C + kci * kc == rows[k, 3 + q]
                    # every absent slot must be zero when the MMA reads it
                    slot = k % S
                    stale = state[slot, q] & ~present & ((1 << G) - 1)
                    assert stale & ~zero == 0
                    state[slot, q] = present
                assert (f >> 16) & 0xF == np_total
                i += nsub
                assert bool(f & LAST) == (i >= len(items))
                k += 1
        assert k == len(rows)


def _sddmm_rowstack_keys(plan, rp, ci, R, C):
    """(block, column in block, row in block) of every 32x32 output tile the
    row-stacked schedule writes, with multiplicity."""
    seen = {}
    for u in plan["unit_table"]:
        row0, nseg = int(u[0]), int(u[1])
        assert row0 % 128 == 0 and 1 <= nseg <= plan["nseg_max"] <= 8
        seg_col = u[4:12]
        blk = u[12:44].reshape(4, 8)
        assert all(seg_col[s] >= 0 and seg_col[s] % 32 == 0 for s in range(nseg))
        assert all(seg_col[s] == -1 for s in range(nseg, 8))
        for q in range(4):
            for s in range(8):
                b = int(blk[q, s])
                if b < 0:
                    continue
                assert s < nseg
                br = (row0 + 32 * q) // R
                assert rp[br] <= b < rp[br + 1]
                assert ci[b] == seg_col[s] // C
                key = (b, int(seg_col[s]) % C, (row0 + 32 * q) % R)
                seen[key] = seen.get(key, 0) + 1
    return seen


def _check_resident_a_runs(plan):
    """Resident-A schedules: in each CTA's list, pad[0] = run << 1 | first
    marks runs of equal row0 (run counting from 0 per CTA) and pad[1] the
    last unit of each run; other schedules leave both words 0."""
    u, cta = plan["unit_table"], plan["cta_begin"]
    if not plan["keep_a"]:
        assert np.all(u[:, 2] == 0) and np.all(u[:, 3] == 0)
        return
    for c in range(len(cta) - 1):
        run = -1
        for i in range(cta[c], cta[c + 1]):
            first = i == cta[c] or u[i, 0] != u[i - 1, 0]
            run += int(first)
            assert u[i, 2] == (run << 1) | int(first)
            last = i == cta[c + 1] - 1 or u[i + 1, 0] != u[i, 0]
            assert u[i, 3] == int(last)


@pytest.mark.parametrize("strategy", ["naive", "dda", "snf"])
@pytest.mark.parametrize("R,C,K", [(32, 32, 256), (64, 32, 96), (32, 96, 64), (512, 64, 128), (32, 32, 512)])
def test_sddmm_rowstack_schedule_covers_every_tile_once(strategy, R, C, K):
    M, N = 4 * max(R, 128), 8 * C
    rng = np.random.default_rng(R * 7 + C)
    rp, ci, _ = rand_bsr(rng, M, N, R, C, 0.4)
    plan = bsp.inspect_sddmm_plan(M, N, R, C, rp, ci, K, bsp.STRATEGIES[strategy])
    assert plan["variant"] == 1
    seen = _sddmm_rowstack_keys(plan, rp, ci, R, C)
    assert len(seen) == int(rp[-1]) * (C // 32) * (R // 32)
    assert all(v == 1 for v in seen.values())
    assert plan["cta_begin"][-1] == plan["units"]
    # the A tile stays resident for CDA and SnF while two 128 x K tiles fit
    assert plan["keep_a"] == int(strategy != "naive" and K <= 256)
    _check_resident_a_runs(plan)


@pytest.mark.parametrize("group_mma", [4, 5])
def test_split_k_cuts_long_units(group_mma):
    """A few very long block-rows (Zipf-like) make split-K worthwhile: the
    planner cuts their units into parts over consecutive step ranges (each at
    least 4 steps), which evens out the CTAs' step counts; opts.group_rows =
    -1 keeps every unit whole."""
    R = C = 32
    M, K, N = 8192, 8192, 128 if group_mma == 4 else 256
    nbr, nbc = M // R, K // C
    rng = np.random.default_rng(17)
    rows = [sorted(rng.choice(nbc, 200 if i < 8 else 6, replace=False)) for i in range(nbr)]
    rp = np.concatenate([[0], np.cumsum([len(r) for r in rows])]).astype(np.int32)
    ci = np.concatenate(rows).astype(np.int32)

    def stats(plan):
        u, cta = plan["unit_table"], plan["cta_begin"]
        steps = u[:, 6] - u[:, 5]
        per = [int(steps[cta[c]:cta[c + 1]].sum()) for c in range(len(cta) - 1)]
        return u, steps, max(per)

    split = bsp.inspect_spmm_plan(M, K, R, C, rp, ci, N, bsp.DDA, opts=bsp.make_opts(group_mma=group_mma))
    whole = bsp.inspect_spmm_plan(M, K, R, C, rp, ci, N, bsp.DDA,
                                  opts=bsp.make_opts(group_mma=group_mma, group_rows=-1))
    u, steps, worst = stats(split)
    uw, _, worst_whole = stats(whole)
    parts = (u[:, 4] & 0xFF) > 1
    assert parts.any() and not ((uw[:, 4] & 0xFF) > 1).any()
    assert steps[parts].min() >= 4
    assert worst < worst_whole


@pytest.mark.parametrize("n_tiles", [0, 1])
def test_sddmm_snf_contiguous_runs_balanced_by_weight(n_tiles):
    """SnF deals contiguous runs of units whose weights are about equal, so a
    row group's A tile is loaded once per CTA run; group_rows = -1 turns the
    resident tile off without changing the schedule."""
    R = C = 32
    M, N, K = 4096, 4096, 128
    rng = np.random.default_rng(5)
    rp, ci, _ = rand_bsr(rng, M, N, R, C, 0.1)
    plan = bsp.inspect_sddmm_plan(M, N, R, C, rp, ci, K, bsp.SNF, opts=bsp.make_opts(n_tiles=n_tiles))
    u, cta = plan["unit_table"], plan["cta_begin"]
    # the CTA lists concatenate to the planner's unit order (row0 nondecreasing)
    assert np.all(np.diff(u[:, 0]) >= 0)
    w = u[:, 1].astype(np.int64) * (K // plan["kc"]) + 2
    loads = np.array([w[cta[c]:cta[c + 1]].sum() for c in range(len(cta) - 1)])
    assert loads.max() - loads.min() <= 2 * w.max()
    a_loads = int((u[:, 2] & 1).sum())
    assert a_loads <= len(np.unique(u[:, 0])) + plan["ctas"]
    _check_resident_a_runs(plan)
    off = bsp.inspect_sddmm_plan(M, N, R, C, rp, ci, K, bsp.SNF,
                                 opts=bsp.make_opts(n_tiles=n_tiles, group_rows=-1))
    assert off["keep_a"] == 0 and np.array_equal(off["cta_begin"], cta)
    assert np.array_equal(off["unit_table"][:, [0, 1]], u[:, [0, 1]])
    assert np.array_equal(off["unit_table"][:, 4:], u[:, 4:])


def test_sddmm_rowstack_repeated_columns_get_their_own_layer():
    R = C = 32
    M, N = 256, 256
    rp = np.array([0, 3, 3, 5, 5, 5, 5, 5, 7], np.int32)
    ci = np.array([2, 2, 5, 1, 1, 7, 7], np.int32)   # repeats in rows 0, 2 and 7
    for n_tiles in (0, 1, 2):
        plan = bsp.inspect_sddmm_plan(M, N, R, C, rp, ci, 64, bsp.NAIVE, opts=bsp.make_opts(n_tiles=n_tiles))
        seen = _sddmm_rowstack_keys(plan, rp, ci, R, C)
        assert len(seen) == int(rp[-1]) and all(v == 1 for v in seen.values())


@pytest.mark.parametrize("strategy", ["naive", "dda"])
@pytest.mark.parametrize("R,C,K", [(32, 32, 256), (64, 32, 96), (32, 96, 64), (512, 64, 128)])
def test_sddmm_schedule_covers_every_segment_once(strategy, R, C, K):
    M, N = 4 * max(R, 128), 8 * C
    rng = np.random.default_rng(R * 7 + C)
    rp, ci, _ = rand_bsr(rng, M, N, R, C, 0.4)
    plan = bsp.inspect_sddmm_plan(M, N, R, C, rp, ci, K, bsp.STRATEGIES[strategy],
                                  opts=bsp.make_opts(group_mma=2))
    assert plan["variant"] == 0
    seen = {}
    Rs = plan["slab"]
    for u in plan["unit_table"]:
        row, r_off, nseg = int(u[0]), int(u[1]), int(u[2])
        assert 1 <= nseg <= 4
        for q in range(nseg):
            b, col = int(u[4 + q]), int(u[8 + q])
            assert rp[row] <= b < rp[row + 1]
            assert col // C == ci[b] and col % 32 == 0
            key = (b, col % C, r_off)
            seen[key] = seen.get(key, 0) + 1
    assert len(seen) == int(rp[-1]) * (C // 32) * (R // Rs)
    assert all(v == 1 for v in seen.values())


def test_planner_rejects_bad_shapes():
    rp = np.zeros(9, np.int32)
    with pytest.raises(bsp.BspError):
        bsp.inspect_spmm_plan(256, 256, 48, 32, np.zeros(256 // 48 + 1, np.int32), [], 128)
    with pytest.raises(bsp.BspError):
        bsp.inspect_spmm_plan(256, 256, 32, 32, rp, [], 100)  # N % 8
    bad = np.array([0, 2, 1, 1, 1, 1, 1, 1, 1], np.int32)  # decreasing row_ptr
    with pytest.raises(bsp.BspError):
        bsp.inspect_spmm_plan(256, 256, 32, 32, bad, [0, 1], 128)


PAIR_OPTS = [dict(group_mma=5), dict(group_mma=5, steps_per_stage=1),
             dict(group_mma=5, no_load_balance=1, producers=2), dict(group_mma=5, max_ctas=20)]


@pytest.mark.parametrize("shape", SHAPES, ids=[f"{s[0]}x{s[1]}x{s[2]}R{s[3]}C{s[4]}p{s[5]}" for s in SHAPES])
@pytest.mark.parametrize("opts", PAIR_OPTS, ids=[str(o) for o in PAIR_OPTS])
def test_pair_schedule_covers_work_exactly_once(shape, opts):
    """CTA-pair plans: CTA 2c+r of pair c holds entries r*G.. of each pair
    unit; both CTAs walk stage lists of equal length; every entry's blocks
    appear once per 256-column chunk, each at the TMA row of its block; an
    absent slot that still holds an older block of that CTA's ring is loaded
    from a box above the A tensor (zero fill), other absent slots are
    skipped, and the leader's descriptor carries the pair's count of loaded
    slots (its barrier's bytes)."""
    M, K, N, R, C, p = shape
    rng = np.random.default_rng(int(M + K + N + R + 1000 * p))
    rp, ci, _ = rand_bsr(rng, M, K, R, C, p)
    plan = bsp.inspect_spmm_plan(M, K, R, C, rp, ci, N, bsp.DDA, opts=bsp.make_opts(**opts))
    assert plan["variant"] == 2 and plan["ctas"] % 2 == 0 and plan["ctas"] <= 148
    units, cta, steps = plan["unit_table"], plan["cta_begin"], plan["step_table"]
    st, cst = plan["stage_table"], plan["cta_stage_begin"]
    G, Rs, kc, nsub = plan["group_rows"], plan["slab"], plan["kc"], plan["nsub"]
    slabs, nkc = R // Rs, C // kc
    assert G * Rs == 128 and plan["step_stride"] == 1 + 2 * G
    FIRST, LAST, EMPTY, TWO = 1 << 24, 1 << 25, 1 << 26, 1 << 27
    seen = {}
    for pc in range(plan["ctas"] // 2):
        lead = range(cta[2 * pc], cta[2 * pc + 1])
        peer = range(cta[2 * pc + 1], cta[2 * pc + 2])
        assert len(lead) == len(peer)
        assert cst[2 * pc + 1] - cst[2 * pc] == cst[2 * pc + 2] - cst[2 * pc + 1]
        presents = [[], []]
        for r, rng_u in enumerate((lead, peer)):
            rows = st[cst[2 * pc + r]:cst[2 * pc + r + 1]]
            S = plan["stages"]
            state = np.full((S, 2), (1 << G) - 1, dtype=np.int64)  # slot contents unknown at start
            k = 0
            for ui in rng_u:
                row0, nent, _, n0, _, sb, se, mask = (int(x) for x in units[ui])
                assert n0 % 256 == 0 and 0 <= nent <= G
                items = [(j, kci) for j in range(sb, se) for kci in range(nkc)]
                if not items:
                    assert rows[k, 0] & (FIRST | LAST | EMPTY) == FIRST | LAST | EMPTY
                    presents[r].append(0)
                    k += 1
                    continue
                i = 0
                while i < len(items):
                    f = int(rows[k, 0])
                    n_in = 2 if f & TWO else 1
                    assert n_in <= nsub and bool(f & FIRST) == (i == 0) and not f & EMPTY
                    assert rows[k, 1] == (n0 // 64 + 2 * r if N % 64 == 0 else n0 + 128 * r)
                    n_present = 0
                    for q in range(n_in):
                        j, kci = items[i + q]
                        assert rows[k, 3 + q] == steps[j, 0] * C + kci * kc
                        load = (f >> (4 * q)) & 0xF
                        assert (f >> (8 + 4 * q)) & 0xF == 0
                        slot = k % S
                        present = 0
                        for g in range(4):
                            ay = int(rows[k, 5 + 4 * q + g])
                            b = int(steps[j, 1 + r * G + g]) if g < G else -1
                            if g < nent and b >= 0:
                                present |= 1 << g
                                assert (load >> g) & 1
                                assert ci[b] == steps[j, 0] and rp[(row0 + g) // slabs] <= b < rp[(row0 + g) // slabs + 1]
                                assert ay == b * R + ((row0 + g) % slabs) * Rs
                                key = (b, (row0 + g) % slabs, kci, n0)
                                seen[key] = seen.get(key, 0) + 1
                            elif (load >> g) & 1:
                                # stale slot: a zero box, and only where the ring slot held a block
                                assert ay == -Rs and (state[slot, q] >> g) & 1
                            else:
                                assert ay == -1 and not (g < G and (state[slot, q] >> g) & 1)
                        n_present += bin(load).count("1")
                        state[slot, q] = present
                    presents[r].append(n_present)
                    i += n_in
                    assert bool(f & LAST) == (i >= len(items))
                    k += 1
            assert k == len(rows)
        lead_rows = st[cst[2 * pc]:cst[2 * pc + 1]]
        for k in range(len(lead_rows)):
            assert (int(lead_rows[k, 0]) >> 16) & 0x1F == presents[0][k] + presents[1][k]
    assert len(seen) == int(rp[-1]) * slabs * nkc * ((N + 255) // 256)
    assert all(v == 1 for v in seen.values())
    # split-K parts: each CTA's partial has its own workspace slot (rank r of
    # a pair unit cut into n parts uses slots r_off .. r_off + n - 1)
    slots = [int(u[2]) + ((int(u[4]) >> 8) & 0xFF) for u in units if (int(u[4]) & 0xFF) > 1]
    assert len(slots) == len(set(slots))
    assert all((int(u[4]) & 0xFF) >= 1 for u in units)


def test_dda_picks_pair_kernel_only_where_it_pays():
    """Dense-enough patterns go to the CTA-pair kernel, sparse ones stay on
    the single-CTA kernel (the pair's wider column unions cost more there)."""
    for p, want in [(0.05, 1), (0.1, 1), (0.25, 2), (0.5, 2)]:
        rng = np.random.default_rng(77)
        rp, ci, _ = rand_bsr(rng, 4096, 4096, 32, 32, p)
        plan = bsp.inspect_spmm_plan(4096, 4096, 32, 32, rp, ci, 4096, bsp.DDA)
        assert plan["variant"] == want, (p, plan["variant"])


def test_large_b_runs_tile_by_tile():
    """When B (K x N bf16) exceeds 64 MiB the row-stacked plan deals its units
    in column-tile order (each CTA's list has nondecreasing n0), so that the
    CTAs share one B panel in L2 at a time; a B that fits keeps the
    serpentine deal (tiles interleaved on a CTA)."""
    R = C = 32
    rng = np.random.default_rng(23)
    M, K = 16384, 32768
    rp, ci, _ = rand_bsr(rng, M, K, R, C, 0.005)
    for N, tile_major in ((2048, True), (1024, False)):
        plan = bsp.inspect_spmm_plan(M, K, R, C, rp, ci, N, bsp.DDA, opts=bsp.make_opts(group_mma=4))
        u, cta = plan["unit_table"], plan["cta_begin"]
        ordered = all(np.all(np.diff(u[cta[c]:cta[c + 1], 3]) >= 0) for c in range(len(cta) - 1))
        assert ordered == tile_major, N


TW_MMA = (1 << 8, 1 << 9)
TW_FIRST = (1 << 16, 1 << 18)
TW_LAST = (1 << 17, 1 << 19)
TW_EMPTY = 1 << 20
TWIN_SHAPES = [(1024, 1024, 512, 32, 32, 0.1), (2048, 1024, 256, 32, 32, 0.5), (800, 512, 384, 32, 32, 0.3),
               (1024, 1024, 256, 64, 32, 0.2), (512, 512, 256, 32, 32, 0.0), (4096, 4096, 4096, 32, 32, 0.01)]


@pytest.mark.parametrize("shape", TWIN_SHAPES, ids=[f"{s[0]}x{s[1]}x{s[2]}R{s[3]}p{s[4]}" for s in TWIN_SHAPES])
def test_twin_schedule_multiplies_every_block_once_per_tile(shape):
    """Twin units (variant 3): per CTA, the unit records come as (a, b)
    pairs sharing one step range; replaying each CTA's stage list, every
    block of each unit's entries is loaded into its slot exactly once per
    column tile at a stage where its unit multiplies, each unit's FIRST and
    LAST flags bracket its multiplying stages, and the two CTAs of a pair
    walk the same flags."""
    M, K, N, R, C, p = shape
    rng = np.random.default_rng(int(M + N + 7 * R + 100 * p))
    rp, ci, _ = rand_bsr(rng, M, K, R, C, p, empty_rows=(1,))
    plan = bsp.inspect_spmm_plan(M, K, R, C, rp, ci, N, bsp.DDA, opts=bsp.make_opts(group_mma=6))
    assert plan["variant"] == 3
    units, cta, st, csb = plan["unit_table"], plan["cta_begin"], plan["stage_table"], plan["cta_stage_begin"]
    slabs = R // 32
    loaded = {}
    for c in range(len(cta) - 1):
        r = c % 2
        k = int(csb[c])
        assert (cta[c + 1] - cta[c]) % 2 == 0
        for ui in range(int(cta[c]), int(cta[c + 1]), 2):
            ua, ub = units[ui], units[ui + 1]
            assert ua[5] == ub[5] and ua[6] == ub[6] and ua[3] == ub[3]    # same steps, same tile
            nsteps = max(1, int(ua[6] - ua[5]))
            open_ = [False, False]
            done = [False, False]
            for s in range(nsteps):
                w = st[k + s]
                flags = int(w[0]) & 0xFFFFFFFF
                if c % 2 == 1:   # the pair's CTAs share the flag bits above the slot mask
                    assert (flags & ~0xFF) == (int(st[int(csb[c - 1]) + (k - int(csb[c])) + s][0]) & ~0xFF)
                for x in range(2):
                    if flags & TW_FIRST[x]:
                        assert not open_[x] and not done[x]
                        open_[x] = True
                    if flags & TW_MMA[x]:
                        assert open_[x]
                        u = (ua, ub)[x]
                        for g in range(4):
                            assert (flags >> (4 * x + g)) & 1
                            ay = int(w[4 + 4 * x + g])
                            if ay >= 0:
                                assert g < u[1]
                                blk, slab = divmod(ay, R)
                                e = int(u[0]) + g
                                assert slab == (e % slabs) * 32
                                i = e // slabs
                                assert rp[i] <= blk < rp[i + 1]
                                key = (e, blk, int(u[3]))
                                assert key not in loaded
                                loaded[key] = True
                    if flags & TW_LAST[x]:
                        assert open_[x]
                        open_[x] = False
                        done[x] = True
            assert done == [True, True]
            k += nsteps
    # every (entry slab, block, tile) exactly once
    n_tiles = (N + 255) // 256
    want = {(i * slabs + sl, b, t * 256) for i in range(M // R) for b in range(int(rp[i]), int(rp[i + 1]))
            for sl in range(slabs) for t in range(n_tiles)}
    assert set(loaded) == want
