"""The oracle (my restatement of the reference golden) pinned three ways:
bit-exact against the committed fixtures made by the reference's own golden
(tests/golden/make_golden.py), bit-exact against that golden live when
oracle/_ref was built here, and against closed-form known answers of the
reference's own tests."""
import glob
import os

import numpy as np
import pytest

import oracle

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
# fixtures storing their inputs; the reference's structural fixtures (frozen
# patterns, hang and deadlock repros) store a seed instead and are pinned below
SEEDED = ("spmm_frozen_profiling_suite", "spmm_test_random_hang", "spmm_test_random_hang_v2",
          "sddmm_deadlock_sweepK_0")
FIXTURES = sorted(f for f in glob.glob(os.path.join(GOLDEN, "*.npz"))
                  if os.path.basename(f)[:-4] not in SEEDED)


def test_fixtures_present():
    names = {os.path.basename(f)[:-4] for f in FIXTURES}
    assert {"spmm_config1", "spmm_1_block_id", "sddmm_identity_mask_R32", "sddmm_random_p15"} <= names
    assert {"spgemm_rand_32", "spgemm_repeats", "spgemm_fill_diag"} <= names
    assert len(FIXTURES) >= 30


@pytest.mark.parametrize("path", FIXTURES, ids=[os.path.basename(f)[:-4] for f in FIXTURES])
def test_oracle_reproduces_reference_fixture(path):
    z = np.load(path)
    if str(z["kind"]) == "spgemm":
        Ra, Ca, Cb, Wb = (int(z[k]) for k in ("Ra", "Ca", "Cb", "Wb"))
        orp, oci, out = oracle.spgemm_bf16(z["a_indptr"], z["a_indices"], z["a_values"], Ra, Ca,
                                           z["b_indptr"], z["b_indices"], z["b_values"], Cb, Wb // Cb)
        assert np.array_equal(orp, z["out_indptr"]) and np.array_equal(oci, z["out_indices"])
        assert np.array_equal(out, z["out"])
        return
    H, W, R, C = (int(z[k]) for k in ("H", "W", "R", "C"))
    ip, ix = z["indptr"], z["indices"]
    if str(z["kind"]) == "spmm":
        N = int(z["N"])
        out = oracle.spmm_bf16(ip, ix, z["values"], H, W, R, C, z["B"], N, threads=2)
        assert np.array_equal(out, z["out"])
        f = oracle.spmm_f32(ip, ix, oracle.bf16_to_f32(z["values"]), H, W, R, C,
                            oracle.bf16_to_f32(z["B"]), N)
        assert np.array_equal(f, z["out_f32"])
    else:
        K = int(z["K"])
        out = oracle.sddmm_bf16(ip, ix, z["mask"], H, W, R, C, z["A"], z["B"], K, threads=2)
        assert np.array_equal(out, z["out"])
        f = oracle.sddmm_f32(ip, ix, oracle.bf16_to_f32(z["mask"]), H, W, R, C,
                             oracle.bf16_to_f32(z["A"]), oracle.bf16_to_f32(z["B"]), K)
        assert np.array_equal(f, z["out_f32"])


def test_known_answers():
    """Closed forms of block_spmm/inc/test_suite.hpp test_1_block_* (32x32)."""
    z = np.load(os.path.join(GOLDEN, "spmm_1_block_id.npz"))
    assert np.array_equal(oracle.bf16_to_f32(z["out"]).reshape(32, 32), np.eye(32, dtype=np.float32))
    z = np.load(os.path.join(GOLDEN, "spmm_1_block_uniform.npz"))
    assert np.all(oracle.bf16_to_f32(z["out"]) == 32.0)
    z = np.load(os.path.join(GOLDEN, "spmm_1_block_arange.npz"))
    a = oracle.bf16_to_f32(z["values"]).reshape(32, 32).astype(np.float64)
    expect = np.repeat(a.sum(1, keepdims=True), 32, axis=1)
    got = oracle.bf16_to_f32(z["out"]).reshape(32, 32)
    assert np.allclose(got, expect, rtol=2 ** -7)
    # SDDMM identity mask: each output block is diag(A B) on that block
    z = np.load(os.path.join(GOLDEN, "sddmm_identity_mask_R32.npz"))
    A = oracle.bf16_to_f32(z["A"]).astype(np.float64)
    B = oracle.bf16_to_f32(z["B"]).astype(np.float64)
    full = A @ B
    out = oracle.bf16_to_f32(z["out"]).reshape(-1, 32, 32)
    for b in range(out.shape[0]):
        d = np.diag(np.diag(full[b * 32:(b + 1) * 32, b * 32:(b + 1) * 32]))
        assert np.allclose(out[b], d, rtol=2 ** -7, atol=0)


@pytest.mark.skipif(not oracle.ref_available(), reason="reference golden not built here")
@pytest.mark.parametrize("R,C,N,p", [(32, 32, 256, 0.1), (64, 32, 96, 0.3), (32, 64, 40, 0.5), (96, 64, 64, 0.4)])
def test_oracle_matches_reference_golden_live(R, C, N, p):
    rng = np.random.default_rng(R * C + N)
    H, W = 8 * R, 8 * C
    occ = rng.random((H // R, W // C)) < p
    ip = np.concatenate([[0], np.cumsum(occ.sum(1))]).astype(np.int32)
    ix = np.nonzero(occ)[1].astype(np.int32)
    vals = oracle.f32_to_bf16(rng.uniform(-1, 1, ix.size * R * C).astype(np.float32))
    B = oracle.f32_to_bf16(rng.uniform(-1, 1, (W, N)).astype(np.float32))
    assert np.array_equal(oracle.spmm_bf16(ip, ix, vals, H, W, R, C, B, N),
                          oracle.ref_spmm_bf16(ip, ix, vals, H, W, R, C, B, N))
    K = 64
    A = oracle.f32_to_bf16(rng.normal(0, 1, (H, K)).astype(np.float32))
    Bs = oracle.f32_to_bf16(rng.normal(0, 1, (K, W)).astype(np.float32))
    g, oip, oix = oracle.ref_sddmm_bf16(ip, ix, vals, H, W, R, C, A, Bs, K)
    assert np.array_equal(oracle.sddmm_bf16(ip, ix, vals, H, W, R, C, A, Bs, K), g)
    assert np.array_equal(oip, ip) and np.array_equal(oix, ix)


@pytest.mark.skipif(not oracle.ref_available(), reason="reference golden not built here")
@pytest.mark.parametrize("Ra,Ca,Cb,pa,pb", [(32, 32, 32, 0.3, 0.3), (64, 32, 32, 0.5, 0.2),
                                            (32, 64, 128, 0.2, 0.6), (128, 32, 64, 0.4, 0.4)])
def test_spgemm_oracle_matches_reference_golden_live(Ra, Ca, Cb, pa, pb):
    rng = np.random.default_rng(Ra + 7 * Ca + 13 * Cb)
    nbr, nbk, nbc = 6, 5, 7
    occ_a = rng.random((nbr, nbk)) < pa
    occ_b = rng.random((nbk, nbc)) < pb
    arp = np.concatenate([[0], np.cumsum(occ_a.sum(1))]).astype(np.int32)
    aci = np.nonzero(occ_a)[1].astype(np.int32)
    brp = np.concatenate([[0], np.cumsum(occ_b.sum(1))]).astype(np.int32)
    bci = np.nonzero(occ_b)[1].astype(np.int32)
    av = oracle.f32_to_bf16(rng.uniform(-1, 1, aci.size * Ra * Ca).astype(np.float32))
    bv = oracle.f32_to_bf16(rng.uniform(-1, 1, bci.size * Ca * Cb).astype(np.float32))
    got = oracle.spgemm_bf16(arp, aci, av, Ra, Ca, brp, bci, bv, Cb, nbc)
    ref = oracle.ref_spgemm_bf16(arp, aci, av, nbr * Ra, nbk * Ca, Ra, Ca, brp, bci, bv, nbc * Cb, Cb)
    for g, r in zip(got, ref):
        assert np.array_equal(g, r)


def test_spgemm_oracle_closed_form():
    """Block-diagonal identity A times B returns B's blocks on B's pattern."""
    rng = np.random.default_rng(3)
    n = 4
    arp = np.arange(n + 1, dtype=np.int32)
    aci = np.arange(n, dtype=np.int32)
    av = oracle.f32_to_bf16(np.tile(np.eye(32, dtype=np.float32).ravel(), n))
    occ = rng.random((n, 5)) < 0.5
    brp = np.concatenate([[0], np.cumsum(occ.sum(1))]).astype(np.int32)
    bci = np.nonzero(occ)[1].astype(np.int32)
    bv = oracle.f32_to_bf16(rng.uniform(-1, 1, bci.size * 32 * 32).astype(np.float32))
    orp, oci, out = oracle.spgemm_bf16(arp, aci, av, 32, 32, brp, bci, bv, 32, 5)
    assert np.array_equal(orp, brp) and np.array_equal(oci, bci) and np.array_equal(out, bv)


@pytest.mark.skipif(not oracle.ref_available(), reason="reference golden not built here")
def test_attention_chain_restatement_matches_reference_goldens():
    """The attention chain through the restated goldens equals the chain
    through the reference's own compiled goldens, bit for bit."""
    rng = np.random.default_rng(12)
    S, d = 256, 64
    occ = rng.random((S // 32, S // 32)) < 0.4
    rp = np.concatenate([[0], np.cumsum(occ.sum(1))]).astype(np.int32)
    ci = np.nonzero(occ)[1].astype(np.int32)
    Q, K, V = (oracle.f32_to_bf16(rng.normal(0, 1, (S, d)).astype(np.float32)) for _ in range(3))
    a = oracle.attention_bf16(rp, ci, S, d, Q, K, V, 0.125)
    b = oracle.attention_bf16(rp, ci, S, d, Q, K, V, 0.125, use_ref=True)
    assert np.array_equal(a, b)


def test_bf16_rounding_is_nearest_even():
    x = np.array([1.0, 1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, -2.5, np.inf, 3.0e38], np.float32)
    b = oracle.f32_to_bf16(x)
    assert oracle.bf16_to_f32(b)[0] == 1.0
    assert oracle.bf16_to_f32(b)[1] == 1.0           # tie to even
    assert oracle.bf16_to_f32(b)[2] == 1.0 + 2 ** -6  # tie to even (up)
    assert oracle.bf16_to_f32(b)[3] == -2.5
    assert np.isinf(oracle.bf16_to_f32(b)[4])


# ---- the reference's structural fixtures (patterns read from its headers) ----
def _sub_rows(ip, ix, vals, R, C, blocks):
    sub_ip, sub_ix, sub_v = [0], [], []
    vv = vals.reshape(-1, R * C)
    for b in blocks:
        sub_ix.append(ix[ip[b]:ip[b + 1]])
        sub_v.append(vv[ip[b]:ip[b + 1]])
        sub_ip.append(sub_ip[-1] + int(ip[b + 1] - ip[b]))
    return (np.array(sub_ip, np.int32), np.concatenate(sub_ix).astype(np.int32),
            np.concatenate(sub_v).reshape(-1))


def test_rand_fill_restates_reference_generator():
    """oracle.rand_fill draws what the reference's RAND content kind draws
    after srand(seed) (live against the compiled reference generator when
    built here, and against the first values stored in the fixtures)."""
    _, s = oracle.rand_fill(42, 0, 4096)
    z = np.load(os.path.join(GOLDEN, "spmm_frozen_profiling_suite.npz"))
    tag = sorted({k.split("__")[0] for k in z.files if "__" in k})[0]
    assert np.array_equal(oracle.f32_to_bf16(s)[:256], z[f"{tag}__b_head"])
    if oracle.ref_available():
        assert np.array_equal(s, oracle.ref_generate_dense(64, 64, oracle.RAND, seed=42).ravel())


FROZEN_PIN = ["M8192_N8192_K8192_R32_C32_dppm30", "M8192_N8192_K8192_R32_C32_dppm3000",
              "M8192_N8192_K8192_R64_C64_dppm600", "M8192_N8192_K8192_R128_C128_dppm50000",
              "M8192_N8192_K512_R256_C256_dppm100000", "M8192_N1024_K8192_R256_C256_dppm100000"]


@pytest.mark.parametrize("tag", FROZEN_PIN)
def test_oracle_reproduces_frozen_pattern_golden(tag):
    """Bit-exact: the oracle on the sampled rows and columns of a frozen
    profiling pattern equals the reference golden stored for them."""
    z = np.load(os.path.join(GOLDEN, "spmm_frozen_profiling_suite.npz"))
    assert len({k.split("__")[0] for k in z.files if "__" in k}) == 36
    M, N, K, R, C, _ = (int(x) for x in z[f"{tag}__shape"])
    ip, ix, rows, cols = z[f"{tag}__indptr"], z[f"{tag}__indices"], z[f"{tag}__rows"], z[f"{tag}__cols"]
    _, s = oracle.rand_fill(int(z["b_seed"]), 0, K * N)
    B = oracle.f32_to_bf16(s.reshape(K, N)[:, cols])
    vals = np.full(ix.size * R * C, 0x3F80, np.uint16)
    blocks = np.unique(rows // R)
    sip, six, sv = _sub_rows(ip, ix, vals, R, C, blocks)
    out = oracle.spmm_bf16(sip, six, sv, blocks.size * R, K, R, C, B, cols.size, threads=4)
    pos = {int(b): i for i, b in enumerate(blocks)}
    sel = np.array([pos[int(r) // R] * R + int(r) % R for r in rows])
    assert np.array_equal(out[sel], z[f"{tag}__out"])


@pytest.mark.parametrize("name", ["spmm_test_random_hang", "spmm_test_random_hang_v2"])
def test_oracle_reproduces_hang_pattern_golden(name):
    z = np.load(os.path.join(GOLDEN, name + ".npz"))
    M, K, R, C, N = (int(z[k]) for k in ("H", "W", "R", "C", "N"))
    u, s = oracle.rand_fill(int(z["seed"]), z["indices"].size * R * C, K * N)
    out = oracle.spmm_bf16(z["indptr"], z["indices"], oracle.f32_to_bf16(u), M, K, R, C,
                           oracle.f32_to_bf16(s).reshape(K, N), N, threads=4)
    assert np.array_equal(out[np.ix_(z["rows"], z["cols"])], z["out"])


def test_oracle_reproduces_sddmm_deadlock_golden():
    z = np.load(os.path.join(GOLDEN, "sddmm_deadlock_sweepK_0.npz"))
    M, N, R, C, K = (int(z[k]) for k in ("H", "W", "R", "C", "K"))
    ip, ix = z["indptr"], z["indices"]
    nb = ix.size
    _, s = oracle.rand_fill(int(z["seed"]), 0, nb * R * C + M * K + K * N)
    mask = oracle.f32_to_bf16(s[:nb * R * C] * np.float32(2.0 ** int(z["mask_scale_log2"])))
    A = oracle.f32_to_bf16(s[nb * R * C:nb * R * C + M * K]).reshape(M, K)
    B = oracle.f32_to_bf16(s[nb * R * C + M * K:]).reshape(K, N)
    # only the sampled blocks' block-rows
    brs = np.unique(np.searchsorted(ip, z["blocks"], side="right") - 1)
    out = np.zeros(nb * R * C, np.uint16)
    for b in brs:
        o = oracle.sddmm_bf16(ip, ix, mask, M, N, R, C, A, B, K, threads=4, rows=(int(b), int(b) + 1))
        out[ip[b] * R * C:ip[b + 1] * R * C] = o[ip[b] * R * C:ip[b + 1] * R * C]
    got = out.reshape(nb, R, C)[z["blocks"]][:, z["rows"]][:, :, z["cols"]]
    assert np.array_equal(got, z["out"])
