"""CPU checkers for the block-sparse SpMM / SDDMM path.

TEST INFRASTRUCTURE ONLY.  Only tests/, ``__graft_entry__.smoke()`` and the
cpu_baseline / reference legs of ``bench.py`` import this package, and only as
the checker or the timed CPU baseline.  The product library never does.

Two checkers live here:

* ``liboracle.so`` (built from ``bsp_oracle.c``): my restatement of the
  reference golden, reference lines cited in the C source.
* ``_ref/libref_golden.so``: the reference's own golden
  (``sparse_common/bsr_matrix.hpp``), compiled from the reference sources in
  place by ``oracle/Makefile``.  It pins the restatement; it is optional at run
  time (absent when the reference sources were not available to build it).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_ORACLE_SO = os.path.join(HERE, "liboracle.so")
_REF_SO = os.path.join(HERE, "_ref", "libref_golden.so")

_i64 = ctypes.c_int64
_i32 = ctypes.c_int32
_p = ctypes.c_void_p

_lib = None
_ref = None


def build(quiet: bool = True) -> None:
    """Compile the checkers (oracle/Makefile)."""
    out = subprocess.run(["make", "-C", HERE], capture_output=True, text=True)
    if out.returncode != 0:
        raise RuntimeError("oracle build failed:\n" + out.stdout + out.stderr)
    if not quiet:
        print(out.stdout)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_ORACLE_SO):
            build()
        _lib = ctypes.CDLL(_ORACLE_SO)
        P, I = _p, _i64
        _lib.bsp_oracle_spmm_bf16_mt.argtypes = [I, I, I, I, P, P, P, I, P, P, I, I, _i32]
        _lib.bsp_oracle_spmm_f32.argtypes = [I, I, I, I, P, P, P, I, P, P, I, I]
        _lib.bsp_oracle_sddmm_bf16_mt.argtypes = [I, I, I, I, P, P, P, I, P, P, P, I, I, _i32]
        _lib.bsp_oracle_sddmm_f32.argtypes = [I, I, I, I, P, P, P, I, P, P, P, I, I]
        _lib.bsp_oracle_serpentine.argtypes = [I, I, P, P]
        _lib.bsp_oracle_spgemm_symbolic.argtypes = [I, I, P, P, P, P, P, P]
        _lib.bsp_oracle_spgemm_symbolic.restype = _i64
        _lib.bsp_oracle_spgemm_bf16.argtypes = [I, I, I, I, P, P, P, P, P, P, P, P, P]
        _lib.bsp_oracle_rand_fill.argtypes = [ctypes.c_uint32, I, P, I, P]
    return _lib


def ref_available() -> bool:
    return os.path.exists(_REF_SO)


def ref():
    """The reference's own golden (None when it was not built)."""
    global _ref
    if _ref is None and ref_available():
        _ref = ctypes.CDLL(_REF_SO)
        P, I = _p, _i64
        _ref.ref_spmm_bf16.argtypes = [I, I, I, I, I, P, P, P, I, P, P]
        _ref.ref_omp_spmm_bf16.argtypes = [I, I, I, I, I, P, P, P, I, P, P]
        _ref.ref_spmm_f32.argtypes = [I, I, I, I, I, P, P, P, I, P, P]
        _ref.ref_sddmm_bf16.argtypes = [I, I, I, I, I, P, P, P, I, P, P, P, P, P]
        _ref.ref_sddmm_f32.argtypes = [I, I, I, I, I, P, P, P, I, P, P, P]
        _ref.ref_pcc_bf16.argtypes = [P, P, I]
        _ref.ref_pcc_bf16.restype = ctypes.c_float
        _ref.ref_bsr_generate.argtypes = [I, I, I, I, I, _i32, _i32, ctypes.c_uint32, P, P, P]
        _ref.ref_bsr_generate.restype = _i64
        _ref.ref_dense_generate.argtypes = [I, I, _i32, ctypes.c_uint32, P]
        _ref.ref_spmm_bf16_timed.argtypes = [I, I, I, I, P, P, P, I, P, I, I, _i32, _i32]
        _ref.ref_spmm_bf16_timed.restype = ctypes.c_double
        _ref.ref_sddmm_bf16_timed.argtypes = [I, I, I, I, P, P, P, I, P, P, I, I, _i32, _i32]
        _ref.ref_sddmm_bf16_timed.restype = ctypes.c_double
        _ref.ref_spgemm_bf16.argtypes = [I, I, I, I, I, P, P, P, I, I, I, P, P, P, I, P, P, P]
        _ref.ref_spgemm_bf16.restype = _i64
    return _ref


def _ptr(a):
    return None if a is None else a.ctypes.data


def _c(a, dt):
    return None if a is None else np.ascontiguousarray(a, dtype=dt)


# ---- bf16 helpers (raw uint16 bit patterns) -------------------------------

def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even f32 -> bf16 bits (NaN kept quiet)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf16_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# ---- the restatement -------------------------------------------------------

def spmm_bf16(indptr, indices, data, H, W, R, C, B, N, threads=None, rows=None):
    """C = A_bsr @ B, bf16 bits in / out (see bsp_oracle_spmm_bf16)."""
    indptr, indices = _c(indptr, np.int32), _c(indices, np.int32)
    data, B = _c(data, np.uint16), _c(B, np.uint16)
    out = np.zeros((H, N), dtype=np.uint16)
    r0, r1 = rows if rows is not None else (0, H // R)
    lib().bsp_oracle_spmm_bf16_mt(H, W, R, C, _ptr(indptr), _ptr(indices), _ptr(data), N,
                                  _ptr(B), _ptr(out), r0, r1, threads or os.cpu_count() or 1)
    return out


def spmm_f32(indptr, indices, data, H, W, R, C, B, N):
    indptr, indices = _c(indptr, np.int32), _c(indices, np.int32)
    data, B = _c(data, np.float32), _c(B, np.float32)
    out = np.zeros((H, N), dtype=np.float32)
    lib().bsp_oracle_spmm_f32(H, W, R, C, _ptr(indptr), _ptr(indices), _ptr(data), N, _ptr(B),
                              _ptr(out), 0, H // R)
    return out


def sddmm_bf16(indptr, indices, mask_data, H, W, R, C, A, B, K, threads=None, rows=None):
    """out_blocks = mask (.) (A @ B) on the mask pattern, bf16 bits (only the
    blocks of block-rows ``rows`` = (r0, r1) are computed when given)."""
    indptr, indices = _c(indptr, np.int32), _c(indices, np.int32)
    mask_data = None if mask_data is None else _c(mask_data, np.uint16)
    A, B = _c(A, np.uint16), _c(B, np.uint16)
    nnzb = int(indptr[-1])
    out = np.zeros(nnzb * R * C, dtype=np.uint16)
    r0, r1 = rows if rows is not None else (0, H // R)
    lib().bsp_oracle_sddmm_bf16_mt(H, W, R, C, _ptr(indptr), _ptr(indices), _ptr(mask_data), K,
                                   _ptr(A), _ptr(B), _ptr(out), r0, r1,
                                   threads or os.cpu_count() or 1)
    return out


def sddmm_f32(indptr, indices, mask_data, H, W, R, C, A, B, K):
    indptr, indices = _c(indptr, np.int32), _c(indices, np.int32)
    mask_data, A, B = _c(mask_data, np.float32), _c(A, np.float32), _c(B, np.float32)
    nnzb = int(indptr[-1])
    out = np.zeros(nnzb * R * C, dtype=np.float32)
    lib().bsp_oracle_sddmm_f32(H, W, R, C, _ptr(indptr), _ptr(indices), _ptr(mask_data), K,
                               _ptr(A), _ptr(B), _ptr(out), 0, H // R)
    return out


def attention_bf16(indptr, indices, S, d, Q, K, V, scale, rows=None, use_ref=False):
    """Block-sparse attention step, the reference chain with a row softmax
    between its two goldens: Sc = sddmm(mask, Q, K^T) with T = float
    (bsr_matrix.hpp:816-857), P = softmax over each row's stored positions of
    scale * Sc (float64, then rounded once to bf16), O = spmm_bfloat16(P, V)
    (bsr_matrix.hpp:692-736).  The mask (S x S, 32 x 32 blocks) is a pattern:
    a column repeated in a row counts once.  Q, K, V: [S, d] bf16 bits.
    Returns O [S, d] bf16 bits (rows of block-rows without blocks are 0).
    ``rows`` = (r0, r1) restricts the work to those block-rows (others 0).
    ``use_ref`` runs the two products through the reference's own compiled
    goldens (oracle/_ref) instead of the restatement."""
    R = 32
    rp = _c(indptr, np.int32)
    ci = _c(indices, np.int32)
    nbr = S // R
    r0, r1 = rows if rows is not None else (0, nbr)
    # the pattern as sets, rows outside [r0, r1) emptied
    sets = [np.unique(ci[rp[i]:rp[i + 1]]) if r0 <= i < r1 else np.zeros(0, np.int32)
            for i in range(nbr)]
    urp = np.concatenate([[0], np.cumsum([len(x) for x in sets])]).astype(np.int32)
    uci = (np.concatenate(sets) if urp[-1] else np.zeros(0, np.int32)).astype(np.int32)
    nnzb = int(urp[-1])
    O = np.zeros((S, d), dtype=np.uint16)
    if nnzb == 0:
        return O
    Qf = bf16_to_f32(_c(Q, np.uint16)).reshape(S, d)
    Kt = np.ascontiguousarray(bf16_to_f32(_c(K, np.uint16)).reshape(S, d).T)
    ones = np.ones(nnzb * R * R, np.float32)
    sd = ref_sddmm_f32 if use_ref else sddmm_f32
    Sc = sd(urp, uci, ones, S, S, R, R, Qf, Kt, d).reshape(nnzb, R, R)
    P = np.zeros_like(Sc)
    for i in range(r0, r1):
        b0, b1 = urp[i], urp[i + 1]
        if b0 == b1:
            continue
        x = Sc[b0:b1].transpose(1, 0, 2).reshape(R, -1).astype(np.float64) * scale
        x -= x.max(axis=1, keepdims=True)
        e = np.exp(x)
        e /= e.sum(axis=1, keepdims=True)
        P[b0:b1] = e.reshape(R, b1 - b0, R).transpose(1, 0, 2)
    Pb = f32_to_bf16(P.astype(np.float32).ravel())
    if use_ref:
        return ref_spmm_bf16(urp, uci, Pb, S, S, R, R, _c(V, np.uint16).reshape(S, d), d)
    return spmm_bf16(urp, uci, Pb, S, S, R, R, _c(V, np.uint16).reshape(S, d), d)


def rand_fill(seed: int, n_unit: int, n_signed: int):
    """(unit, signed) float32 arrays drawn as the reference's generators draw
    them after srand(seed): n_unit values rand()/RAND_MAX, then n_signed values
    of the RAND content kind (see bsp_oracle_rand_fill)."""
    u = np.empty(max(n_unit, 1), np.float32)
    s = np.empty(max(n_signed, 1), np.float32)
    lib().bsp_oracle_rand_fill(seed, n_unit, _ptr(u), n_signed, _ptr(s))
    return u[:n_unit], s[:n_signed]


def serpentine(n: int, parts: int):
    """(owner, slot) per position of the heaviest-first permutation."""
    owner = np.zeros(n, dtype=np.int32)
    slot = np.zeros(n, dtype=np.int32)
    lib().bsp_oracle_serpentine(n, parts, _ptr(owner), _ptr(slot))
    return owner, slot


def spgemm_pattern(a_rp, a_ci, b_rp, b_ci, nbc_b):
    """Block pattern (row_ptr, col_idx) of A_bsr @ B_bsr (bsp_oracle_spgemm_symbolic)."""
    a_rp, a_ci = _c(a_rp, np.int32), _c(a_ci, np.int32)
    b_rp, b_ci = _c(b_rp, np.int32), _c(b_ci, np.int32)
    nbr = a_rp.size - 1
    out_rp = np.zeros(nbr + 1, dtype=np.int32)
    n = int(lib().bsp_oracle_spgemm_symbolic(nbr, nbc_b, _ptr(a_rp), _ptr(a_ci), _ptr(b_rp),
                                             _ptr(b_ci), _ptr(out_rp), None))
    out_ci = np.zeros(max(n, 1), dtype=np.int32)
    lib().bsp_oracle_spgemm_symbolic(nbr, nbc_b, _ptr(a_rp), _ptr(a_ci), _ptr(b_rp), _ptr(b_ci),
                                     _ptr(out_rp), _ptr(out_ci))
    return out_rp, out_ci[:n]


def spgemm_bf16(a_rp, a_ci, a_vals, Ra, Ca, b_rp, b_ci, b_vals, Cb, nbc_b):
    """A_bsr (Ra x Ca blocks) @ B_bsr (Ca x Cb blocks) -> (row_ptr, col_idx, values) in BSR,
    bf16 bits (bsp_oracle_spgemm_bf16)."""
    out_rp, out_ci = spgemm_pattern(a_rp, a_ci, b_rp, b_ci, nbc_b)
    a_rp, a_ci, a_vals = _c(a_rp, np.int32), _c(a_ci, np.int32), _c(a_vals, np.uint16)
    b_rp, b_ci, b_vals = _c(b_rp, np.int32), _c(b_ci, np.int32), _c(b_vals, np.uint16)
    out = np.zeros(max(out_ci.size * Ra * Cb, 1), dtype=np.uint16)
    lib().bsp_oracle_spgemm_bf16(a_rp.size - 1, Ra, Ca, Cb, _ptr(a_rp), _ptr(a_ci), _ptr(a_vals),
                                 _ptr(b_rp), _ptr(b_ci), _ptr(b_vals), _ptr(out_rp), _ptr(out_ci),
                                 _ptr(out))
    return out_rp, out_ci, out[: out_ci.size * Ra * Cb]


# ---- the reference golden (oracle/_ref) -----------------------------------

def ref_spmm_bf16(indptr, indices, data, H, W, R, C, B, N, omp_variant=False):
    r = ref()
    indptr, indices = _c(indptr, np.int32), _c(indices, np.int32)
    data, B = _c(data, np.uint16), _c(B, np.uint16)
    out = np.zeros((H, N), dtype=np.uint16)
    fn = r.ref_omp_spmm_bf16 if omp_variant else r.ref_spmm_bf16
    fn(H, W, R, C, int(indptr[-1]), _ptr(indptr), _ptr(indices), _ptr(data), N, _ptr(B), _ptr(out))
    return out


def ref_spmm_f32(indptr, indices, data, H, W, R, C, B, N):
    r = ref()
    indptr, indices = _c(indptr, np.int32), _c(indices, np.int32)
    data, B = _c(data, np.float32), _c(B, np.float32)
    out = np.zeros((H, N), dtype=np.float32)
    r.ref_spmm_f32(H, W, R, C, int(indptr[-1]), _ptr(indptr), _ptr(indices), _ptr(data), N,
                   _ptr(B), _ptr(out))
    return out


def ref_sddmm_bf16(indptr, indices, mask_data, H, W, R, C, A, B, K):
    """Returns (out_blocks, out_indptr, out_indices) from the reference golden."""
    r = ref()
    indptr, indices = _c(indptr, np.int32), _c(indices, np.int32)
    nnzb = int(indptr[-1])
    if mask_data is None:
        mask_data = np.full(nnzb * R * C, 0x3F80, dtype=np.uint16)  # 1.0
    mask_data, A, B = _c(mask_data, np.uint16), _c(A, np.uint16), _c(B, np.uint16)
    out = np.zeros(nnzb * R * C, dtype=np.uint16)
    oip = np.zeros(H // R + 1, dtype=np.int32)
    oix = np.zeros(max(nnzb, 1), dtype=np.int32)
    r.ref_sddmm_bf16(H, W, R, C, nnzb, _ptr(indptr), _ptr(indices), _ptr(mask_data), K, _ptr(A),
                     _ptr(B), _ptr(out), _ptr(oip), _ptr(oix))
    return out, oip, oix[:nnzb]


def ref_sddmm_f32(indptr, indices, mask_data, H, W, R, C, A, B, K):
    r = ref()
    indptr, indices = _c(indptr, np.int32), _c(indices, np.int32)
    nnzb = int(indptr[-1])
    if mask_data is None:
        mask_data = np.ones(nnzb * R * C, dtype=np.float32)
    mask_data, A, B = _c(mask_data, np.float32), _c(A, np.float32), _c(B, np.float32)
    out = np.zeros(nnzb * R * C, dtype=np.float32)
    r.ref_sddmm_f32(H, W, R, C, nnzb, _ptr(indptr), _ptr(indices), _ptr(mask_data), K, _ptr(A),
                    _ptr(B), _ptr(out))
    return out


def ref_pcc(a_bf16, b_bf16) -> float:
    a, b = _c(a_bf16.ravel(), np.uint16), _c(b_bf16.ravel(), np.uint16)
    return float(ref().ref_pcc_bf16(_ptr(a), _ptr(b), a.size))


FILL_ROW, FILL_COL, FILL_DIAG, FILL_TRIL, FILL_MULTI_DIAG = 1, 2, 3, 4, 5
RAND, UNIFORM, ARANGE, ID = 0, 1, 2, 3


def ref_generate_bsr(H, W, R, C, nblocks, fill, content, seed=42):
    """The reference's own pattern generator; returns (indptr, indices, data_f32)."""
    r = ref()
    n = r.ref_bsr_generate(H, W, R, C, nblocks, fill, content, seed, None, None, None)
    if n < 0:
        raise ValueError("bad generator arguments")
    ip = np.zeros(H // R + 1, dtype=np.int32)
    ix = np.zeros(max(n, 1), dtype=np.int32)
    d = np.zeros(max(n, 1) * R * C, dtype=np.float32)
    r.ref_bsr_generate(H, W, R, C, nblocks, fill, content, seed, _ptr(ip), _ptr(ix), _ptr(d))
    return ip, ix[:n], d[: n * R * C]


def ref_generate_dense(H, W, content, seed=42):
    out = np.zeros((H, W), dtype=np.float32)
    ref().ref_dense_generate(H, W, content, seed, _ptr(out))
    return out


def ref_spmm_timed(indptr, indices, data, H, W, R, C, B, N, rows, threads, reps=1) -> float:
    """Seconds per call of the reference golden over block-rows ``rows``."""
    indptr, indices = _c(indptr, np.int32), _c(indices, np.int32)
    data, B = _c(data, np.uint16), _c(B, np.uint16)
    return float(ref().ref_spmm_bf16_timed(H, W, R, C, _ptr(indptr), _ptr(indices), _ptr(data),
                                           N, _ptr(B), rows[0], rows[1], threads, reps))


def ref_sddmm_timed(indptr, indices, mask_data, H, W, R, C, A, B, K, rows, threads, reps=1) -> float:
    indptr, indices = _c(indptr, np.int32), _c(indices, np.int32)
    nnzb = int(indptr[-1])
    if mask_data is None:
        mask_data = np.full(nnzb * R * C, 0x3F80, dtype=np.uint16)
    mask_data, A, B = _c(mask_data, np.uint16), _c(A, np.uint16), _c(B, np.uint16)
    return float(ref().ref_sddmm_bf16_timed(H, W, R, C, _ptr(indptr), _ptr(indices),
                                            _ptr(mask_data), K, _ptr(A), _ptr(B), rows[0],
                                            rows[1], threads, reps))


def ref_spgemm_bf16(a_rp, a_ci, a_vals, Ha, Wa, Ra, Ca, b_rp, b_ci, b_vals, Wb, Cb):
    """(row_ptr, col_idx, values) of A @ B from the reference's bsr_matrix::spgemm."""
    r = ref()
    a_rp, a_ci, a_vals = _c(a_rp, np.int32), _c(a_ci, np.int32), _c(a_vals, np.uint16)
    b_rp, b_ci, b_vals = _c(b_rp, np.int32), _c(b_ci, np.int32), _c(b_vals, np.uint16)
    args = (Ha, Wa, Ra, Ca, int(a_rp[-1]), _ptr(a_rp), _ptr(a_ci), _ptr(a_vals), Wb, Cb,
            int(b_rp[-1]), _ptr(b_rp), _ptr(b_ci), _ptr(b_vals))
    n = int(r.ref_spgemm_bf16(*args, 0, None, None, None))
    out_rp = np.zeros(Ha // Ra + 1, dtype=np.int32)
    out_ci = np.zeros(max(n, 1), dtype=np.int32)
    out = np.zeros(max(n * Ra * Cb, 1), dtype=np.uint16)
    r.ref_spgemm_bf16(*args, n, _ptr(out_rp), _ptr(out_ci), _ptr(out))
    return out_rp, out_ci[:n], out[: n * Ra * Cb]
