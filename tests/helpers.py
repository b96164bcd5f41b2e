"""Shared helpers for the GPU parity tests (test infrastructure)."""
import numpy as np
import torch


def rel_err(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    scale = max(np.abs(ref).max(), 1e-30)
    return float(np.abs(got - ref).max() / scale)


def assert_close_elementwise(got, ref, rtol, atol_frac):
    """Every element: |got - ref| <= rtol |ref| + atol_frac max|ref| (a per-element relative bound
    with an absolute floor tied to the scale of the result)."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    scale = max(np.abs(ref).max(), 1e-30)
    bound = rtol * np.abs(ref) + atol_frac * scale
    bad = np.abs(got - ref) > bound
    assert not bad.any(), (f"{int(bad.sum())} of {bad.size} elements out of tolerance; worst excess "
                           f"{float((np.abs(got - ref) / bound).max()):.3g}x the bound")


def align_column_signs(A, B, A_ref):
    """Factors are defined up to the sign of each rank-one term (A[:, k], B[:, k]) -> (-A[:, k],
    -B[:, k]): the SVD in the refactoring step may pick either sign. Flip the columns of A and B
    whose A column points away from the reference's."""
    s = np.sign(np.sum(np.asarray(A, np.float64) * np.asarray(A_ref, np.float64), axis=0))
    s[s == 0] = 1.0
    return np.asarray(A) * s, np.asarray(B) * s


def random_edges(rng, n_fixed, n_out, nnz):
    """Distinct (fixed, out) pairs with positive values."""
    keys = rng.choice(n_fixed * n_out, size=nnz, replace=False)
    return (keys // n_out).astype(np.int64), (keys % n_out).astype(np.int64), \
        (0.05 + rng.random(nnz)).astype(np.float32)


def host_csr(fixed_local, out_rows, vals, M):
    """CSR by output row (stable), entries {local fixed row, value bits} as int32 pairs."""
    order = np.argsort(out_rows, kind="stable")
    o = out_rows[order]
    rowptr = np.searchsorted(o, np.arange(M + 1), side="left").astype(np.int32)
    ent = np.stack([fixed_local[order].astype(np.int32),
                    vals[order].astype(np.float32).view(np.int32)], axis=1)
    return rowptr, np.ascontiguousarray(ent)


def to_dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.to(dtype)
    return t.cuda()


def pad(a, Dp):
    out = np.zeros((a.shape[0], Dp), np.float32)
    out[:, :a.shape[1]] = a
    return out
