#!/usr/bin/env python3
"""Generate the golden fixtures in this directory from the REFERENCE's own
CPU golden (oracle/_ref/libref_golden.so, compiled from the reference sources
sparse_common/bsr_matrix.hpp by oracle/Makefile).

Run from the repository root in a container that has the reference sources:
    make -C oracle && python tests/golden/make_golden.py

Cases:
  * the reference's known-answer SpMM tests (block_spmm/inc/test_suite.hpp:
    test_1_block_id / _arange / _uniform: FILL_COL blocks with ID / ARANGE /
    UNIFORM content), built with the reference's own generators;
  * reference fill patterns (FILL_DIAG, FILL_TRIL, FILL_MULTI_DIAG, FILL_ROW,
    FILL_COL) with RAND content after srand(42), as the reference registries do;
  * BASELINE config 1 in full (1024x1024, 32x32 blocks, p = 0.10, N = 256,
    uniform[-1,1], numpy seed 1234);
  * the reference's SDDMM registry shapes (block_sddmm/inc/test_suite.hpp:
    single_block, diagonal_mask, full_mask, identity_mask, nonsquare,
    diagonal_mask_short_k) for R = C = 32 and 64, plus a seeded random mask;
  * SpGEMM (bsr_matrix<T>::spgemm, sparse_common/bsr_matrix.hpp:741-810):
    seeded random patterns for each block-size combination, the reference's
    FILL_DIAG / FILL_TRIL generators, empty block-rows, and rows with
    repeated and unsorted column indices.
Every fixture stores inputs and golden outputs as raw bf16 bit patterns.
`python tests/golden/make_golden.py spgemm` regenerates only the SpGEMM ones.
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
import oracle  # noqa: E402

F = oracle


def save(name, **kw):
    np.savez_compressed(os.path.join(HERE, name + ".npz"), **kw)
    print("wrote", name)


def spmm_case(name, H, W, R, C, N, ip, ix, data_f32, B_f32):
    vals = F.f32_to_bf16(data_f32)
    B = F.f32_to_bf16(B_f32)
    out = F.ref_spmm_bf16(ip, ix, vals, H, W, R, C, B, N)
    out_omp = F.ref_spmm_bf16(ip, ix, vals, H, W, R, C, B, N, omp_variant=True)
    assert np.array_equal(out, out_omp)
    out_f32 = F.ref_spmm_f32(ip, ix, F.bf16_to_f32(vals), H, W, R, C, F.bf16_to_f32(B), N)
    save(name, kind="spmm", H=H, W=W, R=R, C=C, N=N, indptr=ip, indices=ix, values=vals, B=B,
         out=out, out_f32=out_f32)


def sddmm_case(name, H, W, R, C, K, ip, ix, mask_f32, A_f32, B_f32):
    mv = F.f32_to_bf16(mask_f32)
    A = F.f32_to_bf16(A_f32)
    B = F.f32_to_bf16(B_f32)
    out, oip, oix = F.ref_sddmm_bf16(ip, ix, mv, H, W, R, C, A, B, K)
    assert np.array_equal(oip, ip) and np.array_equal(oix, ix)
    out_f32 = F.ref_sddmm_f32(ip, ix, F.bf16_to_f32(mv), H, W, R, C, F.bf16_to_f32(A),
                              F.bf16_to_f32(B), K)
    save(name, kind="sddmm", H=H, W=W, R=R, C=C, K=K, indptr=ip, indices=ix, mask=mv, A=A, B=B,
         out=out, out_f32=out_f32)


def spgemm_case(name, Ha, Wa, Wb, Ra, Ca, Cb, arp, aci, av_f32, brp, bci, bv_f32):
    av, bv = F.f32_to_bf16(av_f32), F.f32_to_bf16(bv_f32)
    orp, oci, out = F.ref_spgemm_bf16(arp, aci, av, Ha, Wa, Ra, Ca, brp, bci, bv, Wb, Cb)
    save(name, kind="spgemm", Ha=Ha, Wa=Wa, Wb=Wb, Ra=Ra, Ca=Ca, Cb=Cb, a_indptr=arp, a_indices=aci,
         a_values=av, b_indptr=brp, b_indices=bci, b_values=bv, out_indptr=orp, out_indices=oci,
         out=out)


def rand_pattern(rng, nbr, nbc, p, empty_rows=()):
    occ = rng.random((nbr, nbc)) < p
    for r in empty_rows:
        occ[r, :] = False
    ip = np.concatenate([[0], np.cumsum(occ.sum(1))]).astype(np.int32)
    return ip, np.nonzero(occ)[1].astype(np.int32)


def spgemm_cases():
    rng = np.random.default_rng(741)
    # seeded random patterns, every block-size family the device path takes
    for name, Ha, Wa, Wb, Ra, Ca, Cb, pa, pb in [
            ("spgemm_rand_32", 512, 384, 448, 32, 32, 32, 0.2, 0.2),
            ("spgemm_rand_64_32_64", 384, 256, 384, 64, 32, 64, 0.3, 0.25),
            ("spgemm_rand_32_64_32", 288, 512, 256, 32, 64, 32, 0.25, 0.3),
            ("spgemm_rand_128_128_32", 384, 512, 192, 128, 128, 32, 0.5, 0.4),
            ("spgemm_rand_32_128_128", 160, 384, 512, 32, 128, 128, 0.4, 0.4)]:
        arp, aci = rand_pattern(rng, Ha // Ra, Wa // Ca, pa, empty_rows=(1,))
        brp, bci = rand_pattern(rng, Wa // Ca, Wb // Cb, pb, empty_rows=(0,))
        spgemm_case(name, Ha, Wa, Wb, Ra, Ca, Cb, arp, aci,
                    rng.uniform(-1, 1, aci.size * Ra * Ca).astype(np.float32), brp, bci,
                    rng.uniform(-1, 1, bci.size * Ca * Cb).astype(np.float32))
    # the reference's own generators (RAND content after srand)
    for name, fa, fb, nb in [("spgemm_fill_diag", F.FILL_DIAG, F.FILL_DIAG, 16),
                             ("spgemm_fill_tril_diag", F.FILL_TRIL, F.FILL_DIAG, 0)]:
        arp, aci, ad = F.ref_generate_bsr(512, 512, 32, 32, nb, fa, F.RAND, seed=42)
        brp, bci, bd = F.ref_generate_bsr(512, 256, 32, 32, 8 if fb == F.FILL_DIAG else nb, fb,
                                          F.RAND, seed=43)
        spgemm_case(name, 512, 512, 256, 32, 32, 32, arp, aci, ad, brp, bci, bd)
    # repeated and unsorted column indices in rows of A and of B
    arp = np.array([0, 3, 3, 7, 9], np.int32)
    aci = np.array([2, 0, 2, 1, 3, 1, 1, 0, 3], np.int32)
    brp = np.array([0, 2, 4, 7, 9], np.int32)
    bci = np.array([1, 1, 2, 0, 4, 3, 4, 0, 2], np.int32)
    spgemm_case("spgemm_repeats", 128, 128, 160, 32, 32, 32, arp, aci,
                rng.uniform(-1, 1, aci.size * 1024).astype(np.float32), brp, bci,
                rng.uniform(-1, 1, bci.size * 1024).astype(np.float32))


def main():
    if not F.ref_available():
        sys.exit("oracle/_ref/libref_golden.so is missing: run `make -C oracle` with the reference sources")
    if sys.argv[1:] == ["spgemm"]:
        spgemm_cases()
        return
    # ---- SpMM known-answer cases (test_suite.hpp:1841-1921) ----
    for name, acontent, bcontent in [("spmm_1_block_id", F.ID, F.ID),
                                     ("spmm_1_block_arange", F.ARANGE, F.UNIFORM),
                                     ("spmm_1_block_uniform", F.UNIFORM, F.UNIFORM)]:
        ip, ix, d = F.ref_generate_bsr(32, 32, 32, 32, 1, F.FILL_COL, acontent)
        B = F.ref_generate_dense(32, 32, bcontent)
        spmm_case(name, 32, 32, 32, 32, 32, ip, ix, d, B)
    # ---- reference fill patterns with RAND content ----
    pats = [("spmm_fill_diag", 512, 512, 32, 32, 16, F.FILL_DIAG, 128),
            ("spmm_fill_tril", 256, 256, 32, 32, 0, F.FILL_TRIL, 64),
            ("spmm_fill_multi_diag", 512, 512, 64, 64, 20, F.FILL_MULTI_DIAG, 96),
            ("spmm_fill_row_nonsquare", 256, 512, 64, 32, 10, F.FILL_ROW, 64),
            ("spmm_fill_col_tall", 512, 256, 128, 32, 6, F.FILL_COL, 32)]
    for name, H, W, R, C, nb, fill, N in pats:
        ip, ix, d = F.ref_generate_bsr(H, W, R, C, nb, fill, F.RAND, seed=42)
        B = F.ref_generate_dense(W, N, F.RAND, seed=43)
        spmm_case(name, H, W, R, C, N, ip, ix, d, B)
    # ---- BASELINE config 1 ----
    rng = np.random.default_rng(1234)
    occ = rng.random((32, 32)) < 0.10
    ip = np.concatenate([[0], np.cumsum(occ.sum(1))]).astype(np.int32)
    ix = np.nonzero(occ)[1].astype(np.int32)
    d = rng.uniform(-1, 1, ix.size * 32 * 32).astype(np.float32)
    B = rng.uniform(-1, 1, (1024, 256)).astype(np.float32)
    spmm_case("spmm_config1", 1024, 1024, 32, 32, 256, ip, ix, d, B)
    # ---- SDDMM registry shapes (block_sddmm/inc/test_suite.hpp:27-107) ----
    for R in (32, 64):
        C = R
        sh = [("single_block", R, C, 1, F.FILL_ROW, F.UNIFORM, R, 2 * C, C, 2 * C),
              ("diagonal_mask", 4 * R, 4 * C, 4, F.FILL_DIAG, F.UNIFORM, 4 * R, 2 * C, 4 * C, 2 * C),
              ("full_mask", 2 * R, 2 * C, 4, F.FILL_ROW, F.UNIFORM, 2 * R, C, 2 * C, C),
              ("identity_mask", 4 * R, 4 * C, 4, F.FILL_DIAG, F.ID, 4 * R, 2 * C, 4 * C, 2 * C),
              ("nonsquare", 8 * R, 4 * C, 8, F.FILL_ROW, F.UNIFORM, 8 * R, 2 * C, 4 * C, 2 * C),
              ("diagonal_mask_shortk", 4 * R, 4 * C, 4, F.FILL_DIAG, F.UNIFORM, 4 * R, C, 4 * C, C)]
        for name, H, W, nb, fill, content, aH, K, bW, bK in sh:
            ip, ix, m = F.ref_generate_bsr(H, W, R, C, nb, fill, content)
            A = F.ref_generate_dense(aH, K, F.ARANGE)
            Bd = F.ref_generate_dense(bK, bW, F.UNIFORM)
            sddmm_case(f"sddmm_{name}_R{R}", H, W, R, C, K, ip, ix, m, A, Bd)
    # seeded random mask (config 3 distributions, small)
    rng = np.random.default_rng(1234 + 3)
    occ = rng.random((16, 16)) < 0.15
    ip = np.concatenate([[0], np.cumsum(occ.sum(1))]).astype(np.int32)
    ix = np.nonzero(occ)[1].astype(np.int32)
    m = np.ones(ix.size * 32 * 32, np.float32)
    A = (rng.normal(0, 1, (512, 256)) / 16).astype(np.float32)
    Bd = (rng.normal(0, 1, (256, 512)) / 16).astype(np.float32)
    sddmm_case("sddmm_random_p15", 512, 512, 32, 32, 256, ip, ix, m, A, Bd)
    spgemm_cases()


if __name__ == "__main__":
    main()
