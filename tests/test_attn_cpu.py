"""Fused attention step, host logic without a GPU: the planner's chunks cover
every distinct (block-row, key block) pair of the mask exactly once, and a
float64 emulation of the kernel's algorithm over that schedule (S per chunk,
masking by the chunk bits, running maximum moved only past a 2^8 growth with
O and the row sum rescaled, P rounded to bf16, O / l at the end) matches the
oracle chain sddmm -> softmax -> spmm."""
import numpy as np
import pytest

import bsp
import oracle


def rand_mask(rng, nbr, p, empty_rows=(), repeats=0):
    rows = []
    for i in range(nbr):
        cols = [] if i in empty_rows else list(np.nonzero(rng.random(nbr) < p)[0])
        for _ in range(repeats):
            if cols:
                cols.append(cols[rng.integers(len(cols))])
        rng.shuffle(cols)
        rows.append(cols)
    rp = np.concatenate([[0], np.cumsum([len(r) for r in rows])]).astype(np.int32)
    ci = np.array([c for r in rows for c in r], dtype=np.int32)
    return rp, ci


def bf16_round(x):
    return oracle.bf16_to_f32(oracle.f32_to_bf16(np.asarray(x, np.float32)))


def emulate(plan, S, d, Q, K, V, scale):
    """The kernel's algorithm over the planned schedule (float64): per unit or
    part, S per chunk, masking by the chunk bits, the lazily moved running
    maximum, bf16 P, O += P V; unsplit units normalise, split units merge
    their parts' (O, m, l) the way the last part does."""
    Qf = oracle.bf16_to_f32(Q).reshape(S, d).astype(np.float64)
    Kf = oracle.bf16_to_f32(K).reshape(S, d).astype(np.float64)
    Vf = oracle.bf16_to_f32(V).reshape(S, d).astype(np.float64)
    O = np.zeros((S, d))
    written = np.zeros(S, np.int32)
    sl2 = scale * np.log2(np.e)
    partials = {}
    for row0, cb, n, n_parts, part, slot0, counter, _ in plan["unit_table"]:
        rows = np.arange(row0, min(row0 + 128, S))
        m = np.full(rows.size, -np.inf)
        lsum = np.zeros(rows.size)
        acc = np.zeros((rows.size, d))
        q = Qf[rows]
        for ch in plan["chunk_table"][cb:cb + n]:
            kb, bits = ch[:4], int(np.uint32(ch[4]))
            keys = np.concatenate([np.arange(32 * b, 32 * b + 32) if b >= 0 else np.full(32, -1) for b in kb])
            Kc = np.where(keys[:, None] >= 0, Kf[np.maximum(keys, 0)], 0.0)
            Vc = np.where(keys[:, None] >= 0, Vf[np.maximum(keys, 0)], 0.0)
            s = (q @ Kc.T) * sl2
            valid = np.zeros((rows.size, 128), bool)
            for i, r in enumerate(rows - row0):
                qq = r // 32
                for sl in range(4):
                    if (bits >> (4 * qq + sl)) & 1:
                        valid[i, 32 * sl:32 * sl + 32] = True
            s = np.where(valid, s, -np.inf)
            mx = s.max(axis=1)
            need = mx > m + 8
            new_m = np.where(need, mx, m)
            with np.errstate(invalid="ignore"):
                alpha = np.where(need, np.where(np.isneginf(m), 0.0, np.exp2(m - new_m)), 1.0)
            acc *= alpha[:, None]
            lsum *= alpha
            m = new_m
            with np.errstate(invalid="ignore"):
                p = np.where(valid, np.exp2(s - m[:, None]), 0.0)
            p = bf16_round(p).astype(np.float64)
            lsum += p.sum(axis=1)
            acc += p @ Vc
        if n_parts == 1:
            inv = np.where(lsum > 0, 1.0 / np.where(lsum > 0, lsum, 1), 0.0)
            O[rows] = acc * inv[:, None]
            written[rows] += 1
            continue
        partials.setdefault(counter, []).append((part, rows, acc, m, lsum))
        if len(partials[counter]) == n_parts:
            parts = sorted(partials.pop(counter), key=lambda t: t[0])
            assert [t[0] for t in parts] == list(range(n_parts))
            M = np.max([t[3] for t in parts], axis=0)
            with np.errstate(invalid="ignore"):
                w = [np.where(np.isneginf(M) | np.isneginf(t[3]), 0.0, np.exp2(t[3] - M)) for t in parts]
            L = sum(wk * t[4] for wk, t in zip(w, parts))
            acc = sum(wk[:, None] * t[2] for wk, t in zip(w, parts))
            inv = np.where(L > 0, 1.0 / np.where(L > 0, L, 1), 0.0)
            O[rows] = acc * inv[:, None]
            written[rows] += 1
    assert not partials
    assert np.all(written == 1)
    return O


def check_schedule(plan, S, rp, ci):
    nbr = S // 32
    seen = set()
    units = {}
    for row0, cb, n, n_parts, part, slot0, counter, _ in plan["unit_table"]:
        units.setdefault(row0, []).append((part, cb, n, n_parts))
    assert len(units) == (nbr + 3) // 4
    for row0, pieces in units.items():
        pieces.sort()
        assert [p_[0] for p_ in pieces] == list(range(len(pieces)))
        assert all(p_[3] == len(pieces) for p_ in pieces) and len(pieces) <= 16
        for a, b in zip(pieces, pieces[1:]):
            assert a[1] + a[2] == b[1]            # consecutive chunk ranges
        cb, n = pieces[0][1], sum(p_[2] for p_ in pieces)
        union = sorted({int(c) for i in range(row0 // 32, min(row0 // 32 + 4, nbr))
                        for c in ci[rp[i]:rp[i + 1]]})
        kbs = [int(k) for ch in plan["chunk_table"][cb:cb + n] for k in ch[:4] if k >= 0]
        assert kbs == union
        assert n == (len(union) + 3) // 4
        for ch in plan["chunk_table"][cb:cb + n]:
            bits = int(np.uint32(ch[4]))
            for q in range(4):
                for sl in range(4):
                    if (bits >> (4 * q + sl)) & 1:
                        i = row0 // 32 + q
                        assert ch[sl] >= 0 and ch[sl] in ci[rp[i]:rp[i + 1]]
                        key = (i, int(ch[sl]))
                        assert key not in seen
                        seen.add(key)
    expect = {(i, int(c)) for i in range(nbr) for c in ci[rp[i]:rp[i + 1]]}
    assert seen == expect
    assert plan["mask_blocks"] == len(expect)
    cta = plan["cta_begin"]
    assert cta[0] == 0 and cta[-1] == plan["units"]


@pytest.mark.parametrize("S,d,p", [(256, 128, 0.3), (480, 64, 0.2), (1024, 128, 0.08), (160, 128, 1.0)])
def test_schedule_and_emulation(S, d, p):
    rng = np.random.default_rng(S + d)
    rp, ci = rand_mask(rng, S // 32, p, empty_rows=(1,))
    plan = bsp.inspect_attn_plan(S, d, rp, ci)
    check_schedule(plan, S, rp, ci)
    Q = oracle.f32_to_bf16(rng.normal(0, 1, (S, d)).astype(np.float32))
    K = oracle.f32_to_bf16(rng.normal(0, 1, (S, d)).astype(np.float32))
    V = oracle.f32_to_bf16(rng.normal(0, 1, (S, d)).astype(np.float32))
    scale = 1 / np.sqrt(d)
    got = emulate(plan, S, d, Q, K, V, scale)
    gold = oracle.bf16_to_f32(oracle.attention_bf16(rp, ci, S, d, Q, K, V, scale)).reshape(S, d)
    err = np.linalg.norm(got - gold) / max(np.linalg.norm(gold), 1e-30)
    assert err < 1e-2
    assert np.all(got[32:64] == 0) and np.all(gold[32:64] == 0)  # empty block-row 1


def test_rescale_path_matches():
    """Scores that grow along the keys force the running-maximum rescale on
    most chunks; the emulated kernel algorithm still matches the oracle."""
    rng = np.random.default_rng(3)
    S, d = 512, 64
    rp, ci = rand_mask(rng, S // 32, 0.6)
    q = np.ones((S, d), np.float32) * 0.5
    k = (np.arange(S, dtype=np.float32)[:, None] / 16.0) * np.ones((1, d), np.float32) / d * 8
    Q, K = oracle.f32_to_bf16(q), oracle.f32_to_bf16(k)
    V = oracle.f32_to_bf16(rng.normal(0, 1, (S, d)).astype(np.float32))
    plan = bsp.inspect_attn_plan(S, d, rp, ci)
    got = emulate(plan, S, d, Q, K, V, 1.0)
    gold = oracle.bf16_to_f32(oracle.attention_bf16(rp, ci, S, d, Q, K, V, 1.0)).reshape(S, d)
    assert np.linalg.norm(got - gold) / np.linalg.norm(gold) < 1e-2


def heavy_mask(rng, nbr):
    """Block-rows 0..3 hold every column; the others a sparse band."""
    rows = [list(range(nbr)) if i < 4 else sorted({max(0, i - 1), i, min(nbr - 1, i + 1)}
                                                  | set(rng.integers(0, nbr, 2).tolist()))
            for i in range(nbr)]
    rp = np.concatenate([[0], np.cumsum([len(r) for r in rows])]).astype(np.int32)
    return rp, np.array([c for r in rows for c in r], np.int32)


@pytest.mark.parametrize("opts,split", [(dict(), True), (dict(n_tiles=1), True), (dict(n_tiles=3), True),
                                        (dict(group_rows=-1), False)])
def test_split_units_schedule_and_merge(opts, split):
    """A heavy unit (or a short part length) is cut into parts; the emulated
    parts merged the way the kernel merges them match the oracle."""
    rng = np.random.default_rng(9)
    S, d = 2048, 64
    rp, ci = heavy_mask(rng, S // 32)
    plan = bsp.inspect_attn_plan(S, d, rp, ci, opts=bsp.make_opts(**opts))
    check_schedule(plan, S, rp, ci)
    assert (plan["parts"] > 0 and plan["split_units"] > 0) == split
    if split and not opts:
        heavy = [u for u in plan["unit_table"] if u[0] == 0]
        assert len(heavy) > 1                      # the 16-chunk unit runs as parts
    Q = oracle.f32_to_bf16(rng.normal(0, 1, (S, d)).astype(np.float32))
    K = oracle.f32_to_bf16(rng.normal(0, 1, (S, d)).astype(np.float32))
    V = oracle.f32_to_bf16(rng.normal(0, 1, (S, d)).astype(np.float32))
    got = emulate(plan, S, d, Q, K, V, 0.125)
    gold = oracle.bf16_to_f32(oracle.attention_bf16(rp, ci, S, d, Q, K, V, 0.125)).reshape(S, d)
    assert np.linalg.norm(got - gold) / np.linalg.norm(gold) < 1e-2


def test_repeated_mask_columns_count_once():
    rng = np.random.default_rng(5)
    S = 256
    rp, ci = rand_mask(rng, S // 32, 0.4, repeats=2)
    plan = bsp.inspect_attn_plan(S, 128, rp, ci)
    check_schedule(plan, S, rp, ci)


def test_bad_arguments():
    rp = np.array([0, 1], np.int32)
    ci = np.array([0], np.int32)
    with pytest.raises(bsp.BspError):
        bsp.inspect_attn_plan(32, 96, rp, ci)      # head size
    with pytest.raises(bsp.BspError):
        bsp.inspect_attn_plan(40, 128, rp, ci)     # S % 32
    with pytest.raises(bsp.BspError):
        bsp.inspect_attn_plan(32, 128, rp, np.array([1], np.int32))  # column out of range
