"""The seeded synthetic stand-ins for the reference's datasets (bench.py), at small sizes on the
CPU: exact nnz of distinct in-range pairs, the configured value distributions, determinism."""
import numpy as np

import bench


def _check_coo(idx, vals, shape, nnz):
    m, n = shape
    assert idx.shape == (2, nnz) and vals.shape == (nnz,)
    assert idx[0].min() >= 0 and idx[0].max() < m and idx[1].min() >= 0 and idx[1].max() < n
    keys = idx[0].astype(np.int64) * n + idx[1]
    assert np.unique(keys).size == nnz  # duplicates merged
    assert np.all(vals > 0) and np.all(np.isfinite(vals))


def test_c4_shape_distinct_pairs_and_values():
    idx, vals, shape = bench.make_c4(seed=4, m=3000, nnz=40000)
    _check_coo(idx, vals, shape, 40000)
    # values log(1 + k) with k = 1 + Geometric(0.3) >= 1
    k = np.expm1(vals.astype(np.float64))
    assert np.allclose(k, np.round(k), atol=1e-3) and k.min() >= 1 - 1e-3
    # power-law degrees: the busiest row holds far more than the mean
    deg = np.bincount(idx[0], minlength=3000)
    assert deg.max() > 10 * deg.mean()


def test_c4_is_deterministic():
    a = bench.make_c4(seed=4, m=2000, nnz=20000)
    b = bench.make_c4(seed=4, m=2000, nnz=20000)
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])


def test_c3_zipf_counts():
    idx, vals, shape = bench.make_c3(seed=3, m=2000, nnz=30000)
    _check_coo(idx, vals, shape, 30000)
    c = np.expm1(vals.astype(np.float64))
    assert c.min() >= 1 - 1e-3


def test_c2_columns_and_value_mass():
    idx, vals, shape = bench.make_c2(seed=2, m=3000, n=784, density=0.19)
    nnz = int(0.19 * 3000 * 784)
    _check_coo(idx, vals, shape, nnz)
    lo, hi = int(0.2 * 784), int(0.8 * 784)
    assert idx[1].min() >= lo and idx[1].max() < hi  # central 60 % of the columns
    assert vals.max() <= 1.0
    frac_big = float(np.mean(vals >= 0.9))
    assert 0.38 < frac_big < 0.5  # 40 % drawn in [0.9, 1] plus the top of the rest
