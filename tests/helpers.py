"""Shared test helpers: seeded BSR generators and the parity comparators."""
import numpy as np

import oracle

TOL = 1e-2  # max relative error bound (bf16 in, fp32 accumulate), per the spec


def rand_bsr(rng, H, W, R, C, p, low=-1.0, high=1.0, empty_rows=()):
    """Independent Bernoulli(p) block occupancy, uniform values, bf16 bits."""
    occ = rng.random((H // R, W // C)) < p
    for r in empty_rows:
        occ[r, :] = False
    rp = np.concatenate([[0], np.cumsum(occ.sum(1))]).astype(np.int32)
    ci = np.nonzero(occ)[1].astype(np.int32)
    vals = oracle.f32_to_bf16(rng.uniform(low, high, ci.size * R * C).astype(np.float32))
    return rp, ci, vals


def rand_dense(rng, H, W, kind="uniform", scale=1.0):
    if kind == "uniform":
        x = rng.uniform(-1, 1, (H, W))
    else:
        x = rng.normal(0, 1, (H, W))
    return oracle.f32_to_bf16((x * scale).astype(np.float32))


def rel_err(dev_f32, gold_f32):
    """Elementwise |d-g| / max(|g|, 1e-3*max|g|) (floor for cancellation)."""
    g = np.asarray(gold_f32, dtype=np.float64)
    d = np.asarray(dev_f32, dtype=np.float64)
    if g.size == 0:
        return np.zeros(0)
    floor = max(1e-3 * np.abs(g).max(), 1e-30)
    return np.abs(d - g) / np.maximum(np.abs(g), floor)


def assert_bf16_close(dev_bits, gold_bits, tol=TOL, what=""):
    d = oracle.bf16_to_f32(np.asarray(dev_bits).ravel())
    g = oracle.bf16_to_f32(np.asarray(gold_bits).ravel())
    assert d.shape == g.shape, (d.shape, g.shape)
    assert np.all(np.isfinite(d)), f"{what}: non-finite values in device output"
    e = rel_err(d, g)
    if e.size:
        k = int(np.argmax(e))
        assert e.max() <= tol, f"{what}: max rel err {e.max():.3e} at {k} (dev {d[k]} gold {g[k]})"


def normwise(dev_f32, gold_f32):
    g = np.asarray(gold_f32, dtype=np.float64).ravel()
    d = np.asarray(dev_f32, dtype=np.float64).ravel()
    n = np.linalg.norm(g)
    return 0.0 if n == 0 else float(np.linalg.norm(d - g) / n)


def pcc(a, b):
    a = np.asarray(a, dtype=np.float64).ravel()
    b = np.asarray(b, dtype=np.float64).ravel()
    if a.std() == 0 or b.std() == 0:
        return 1.0 if np.allclose(a, b) else 0.0
    return float(np.corrcoef(a, b)[0, 1])
