"""Parity of the CUDA kernels (through the C ABI) with the CPU oracle on the same seeded inputs.

Tolerances: 1e-5 in 3xTF32 mode (fp32 accuracy) and the north star's 1e-3 in TF32 mode, both as a
bound on the largest error relative to max|reference| (rel_err) and element by element
(|err| <= tol |ref| + tol max|ref|, assert_close_elementwise); sums and metrics, whose rounding
errors average out, 1e-5 / 1e-4. TF32 mode rounds its operands to the nearest tf32 value, as the
reference's mma.sync path does (cvt.rn.tf32.f32). The CSR builder must be bit-exact.
"""
import numpy as np
import pytest
import torch

from oracle import sumac_oracle as orc
from sumac_b200 import _native, ops
from tests.helpers import assert_close_elementwise, host_csr, pad, random_edges, rel_err, to_dev

pytestmark = pytest.mark.gpu

TOL = {ops.SUMAC_3XTF32: 1e-5, ops.SUMAC_TF32: 1e-3}
SUM_TOL = {ops.SUMAC_3XTF32: 1e-5, ops.SUMAC_TF32: 1e-4}
PRECS = [ops.SUMAC_3XTF32, ops.SUMAC_TF32]



@pytest.mark.parametrize("prec", PRECS)
@pytest.mark.parametrize("D,N,M", [(8, 250, 3000), (13, 77, 1000), (16, 250, 25000), (17, 250, 2000),
                                   (32, 250, 25000), (64, 300, 5000), (128, 250, 2000),
                                   (128, 1000, 3000), (200, 250, 2000), (256, 300, 1500),
                                   (16, 5000, 300), (16, 3, 130)])
def test_relu_bat_c(D, N, M, prec):
    rng = np.random.default_rng(D * 1000 + N)
    A = rng.standard_normal((N, D)).astype(np.float32)
    B = rng.standard_normal((M, D)).astype(np.float32)
    C = rng.standard_normal((N, D)).astype(np.float32)
    Y = ops.relu_bat_c(to_dev(A), to_dev(B), to_dev(C), prec).cpu().numpy()
    _native.raise_device_error(0)
    ref = orc.relu_bat_c(A, B, C)
    assert rel_err(Y, ref) < TOL[prec]
    assert_close_elementwise(Y, ref, TOL[prec], TOL[prec])


@pytest.mark.parametrize("prec", PRECS)
@pytest.mark.parametrize("D", [13, 16, 32, 64, 128, 256])
def test_relu_bat_reduce(D, prec):
    rng = np.random.default_rng(D)
    A = rng.standard_normal((25000, D)).astype(np.float32)
    B = rng.standard_normal((250, D)).astype(np.float32)
    got = ops.relu_bat_reduce(to_dev(A), to_dev(B), prec).cpu().numpy()
    _native.raise_device_error(0)
    ref = orc.relu_bat_reduce(A, B)
    np.testing.assert_allclose(got, ref, rtol=SUM_TOL[prec])


def test_relu_bat_c_golden(golden):
    for tag in "abc":
        g = golden(f"relu_bat_c_{tag}")
        Y = ops.relu_bat_c(to_dev(g["A"]), to_dev(g["B"]), to_dev(g["C"]), ops.SUMAC_3XTF32)
        assert rel_err(Y.cpu().numpy(), g["Y"]) < 1e-5


@pytest.mark.parametrize("prec", PRECS)
@pytest.mark.parametrize("d,N,M,nnz", [(16, 1393, 5000, 20000), (8, 200, 700, 3000),
                                       (32, 300, 4000, 50000), (64, 100, 129, 500),
                                       (128, 300, 700, 3000), (256, 200, 500, 2000)])
def test_masked_product(d, N, M, nnz, prec):
    rng = np.random.default_rng(d + N)
    Dp = ops.padded_rank(d)
    X = rng.standard_normal((M, d)).astype(np.float32)
    F = rng.standard_normal((N, d)).astype(np.float32)
    C = rng.standard_normal((N, d)).astype(np.float32)
    fi, oj, v = random_edges(rng, N, M, nnz)
    rowptr, ent = host_csr(fi, oj, v, M)
    Y = ops.masked_product(to_dev(pad(X, Dp)), to_dev(pad(F, Dp)), to_dev(pad(C, Dp)),
                           to_dev(rowptr), to_dev(ent), prec).cpu().numpy()[:, :d]
    _native.raise_device_error(0)
    ref = orc.masked_residual(F, X, fi, oj, v) @ C.astype(np.float64)
    assert rel_err(Y, ref) < TOL[prec]
    assert_close_elementwise(Y, ref, TOL[prec], TOL[prec])


@pytest.mark.parametrize("m_fixed,M,nb,nnz", [(57, 40, 5, 300), (1000, 777, 13, 40000),
                                              (5000, 3000, 100, 200000), (64, 9, 64, 0),
                                              (300, 5000, 7, 2000), (5000, 800, 300, 30000),
                                              (20000, 9000, 150, 2000000),
                                              (5000, 800, 600, 30000), (6000, 500, 1500, 30000)])
def test_block_csr_bit_exact(m_fixed, M, nb, nnz):
    rng = np.random.default_rng(m_fixed + nb)
    fi, oj, v = random_edges(rng, m_fixed, M, nnz)
    perm = rng.permutation(m_fixed)
    order = np.argsort(oj, kind="stable")
    rowptr, ent = ops.block_csr_build(to_dev(perm), nb, to_dev(fi[order], torch.int32),
                                      to_dev(oj[order], torch.int32), to_dev(v[order]), M)
    rp_ref, loc_ref, v_ref = orc.block_csr(perm, fi, oj, v, nb, M)
    np.testing.assert_array_equal(rowptr.cpu().numpy(), rp_ref)
    if nnz:
        e = ent.cpu().numpy()
        np.testing.assert_array_equal(e[:, 0], loc_ref)
        np.testing.assert_array_equal(e[:, 1], v_ref.view(np.int32))


@pytest.mark.parametrize("prec", PRECS)
# M = 80000: more row tiles than two per SM, as at C4
@pytest.mark.parametrize("d,m_fixed,b,M,nnz", [(16, 5000, 1393, 4000, 30000), (6, 400, 100, 90, 900),
                                               (16, 5000, 1393, 80000, 200000),
                                               (32, 3000, 300, 2500, 20000), (64, 2000, 500, 700, 5000),
                                               (128, 1500, 400, 600, 4000)])
def test_salsa_block_update(d, m_fixed, b, M, nnz, prec):
    rng = np.random.default_rng(d + b)
    Dp = ops.padded_rank(d)
    F = rng.standard_normal((m_fixed, d)).astype(np.float32)
    X = (0.3 * rng.standard_normal((M, d))).astype(np.float32)
    dX = (0.05 * rng.standard_normal((M, d))).astype(np.float32)
    rows = rng.choice(m_fixed, size=b, replace=False)
    li, oj, v = random_edges(rng, b, M, nnz)
    rowptr, ent = host_csr(li, oj, v, M)
    mu, lr, step = 0.7, 0.1, 5
    unbias = np.float32(1.0) - np.float32(mu) ** np.float32(step)
    Xd, dXd = to_dev(pad(X, Dp)), to_dev(pad(dX, Dp))
    ops.salsa_block_update(to_dev(pad(F, Dp)), to_dev(rows), Xd, dXd, d, to_dev(rowptr),
                           to_dev(ent), mu, lr, to_dev(np.array([unbias], np.float32)), prec)
    _native.raise_device_error(0)
    A_I = F[rows].astype(np.float64)
    Bn, dBn = orc.lsq_update(A_I, X, orc.pinv_t(A_I), dX, li, oj, v, mu, float(unbias), lr)
    tol = 1e-4 if prec == ops.SUMAC_3XTF32 else 1e-3
    assert rel_err(dXd.cpu().numpy()[:, :d], dBn) < tol
    assert rel_err(Xd.cpu().numpy()[:, :d], Bn) < tol
    assert_close_elementwise(Xd.cpu().numpy()[:, :d], Bn, tol, tol)
    assert np.all(Xd.cpu().numpy()[:, d:] == 0)


@pytest.mark.parametrize("prec", PRECS)
@pytest.mark.parametrize("d", [16, 32, 64])
def test_salsa_block_update_heavy_rows(d, prec):
    """Power-law rows: the finalize pass hands a row's entries beyond the first eight to the whole
    warp, several rounds of entries per row, with the next round's entries loaded ahead. Rows with
    up to ~300 entries, several heavy rows in one warp's batch and a heavy last row."""
    rng = np.random.default_rng(100 + d)
    m_fixed, b, M = 3000, 400, 1000
    Dp = ops.padded_rank(d)
    F = rng.standard_normal((m_fixed, d)).astype(np.float32)
    X = (0.3 * rng.standard_normal((M, d))).astype(np.float32)
    dX = (0.05 * rng.standard_normal((M, d))).astype(np.float32)
    rows = rng.choice(m_fixed, size=b, replace=False)
    heavy = {0: 300, 1: 170, 2: 41, 3: 9, 5: 64, 7: 33, 8: 97, 123: 250, M - 1: 129}
    li_l, oj_l = [], []
    for r, k in heavy.items():
        li_l.append(rng.choice(b, size=k, replace=False))
        oj_l.append(np.full(k, r))
    li_r, oj_r, _ = random_edges(rng, b, M, 6000)
    keep = ~np.isin(oj_r, list(heavy))
    li = np.concatenate(li_l + [li_r[keep]]).astype(np.int64)
    oj = np.concatenate(oj_l + [oj_r[keep]]).astype(np.int64)
    v = (0.05 + rng.random(li.size)).astype(np.float32)
    rowptr, ent = host_csr(li, oj, v, M)
    mu, lr, step = 0.7, 0.1, 3
    unbias = np.float32(1.0) - np.float32(mu) ** np.float32(step)
    Xd, dXd = to_dev(pad(X, Dp)), to_dev(pad(dX, Dp))
    ops.salsa_block_update(to_dev(pad(F, Dp)), to_dev(rows), Xd, dXd, d, to_dev(rowptr),
                           to_dev(ent), mu, lr, to_dev(np.array([unbias], np.float32)), prec)
    _native.raise_device_error(0)
    A_I = F[rows].astype(np.float64)
    Bn, dBn = orc.lsq_update(A_I, X, orc.pinv_t(A_I), dX, li, oj, v, mu, float(unbias), lr)
    tol = 1e-4 if prec == ops.SUMAC_3XTF32 else 1e-3
    assert rel_err(dXd.cpu().numpy()[:, :d], dBn) < tol
    assert_close_elementwise(Xd.cpu().numpy()[:, :d], Bn, tol, tol)


@pytest.mark.parametrize("prec", PRECS)
@pytest.mark.parametrize("d,m,n,b,nnz", [(8, 2000, 1500, 2000, 40000), (16, 900, 3000, 300, 20000),
                                         (32, 500, 700, 129, 3000), (128, 400, 500, 200, 4000),
                                         (256, 300, 400, 150, 3000)])
def test_gd_block_grad(d, m, n, b, nnz, prec):
    rng = np.random.default_rng(d + m)
    Dp = ops.padded_rank(d)
    A = (0.5 * rng.standard_normal((m, d))).astype(np.float32)
    B = (0.5 * rng.standard_normal((n, d))).astype(np.float32)
    rows = rng.choice(m, size=b, replace=False)
    li, cj, v = random_edges(rng, b, n, nnz)
    rp_b, ent_b = host_csr(li, cj, v, n)        # by column j, entries local i
    rp_a, ent_a = host_csr(cj, li, v, b)        # by local row i, entries j
    gA = torch.zeros((m, Dp), device="cuda")
    gB = torch.zeros((n, Dp), device="cuda")
    ops.gd_block_grad(to_dev(pad(A, Dp)), to_dev(pad(B, Dp)), d, to_dev(rows), to_dev(rp_b),
                      to_dev(ent_b), to_dev(rp_a), to_dev(ent_a), gA, gB, 0, prec)
    _native.raise_device_error(0)
    _, gAI_ref, gB_ref = orc.gd_block_grad(A[rows], B, li, cj, v)
    tol = TOL[prec]
    assert rel_err(gA.cpu().numpy()[rows, :d], gAI_ref) < tol
    assert rel_err(gB.cpu().numpy()[:, :d], gB_ref) < tol
    assert_close_elementwise(gB.cpu().numpy()[:, :d], gB_ref, tol, tol)
    mask = np.ones(m, bool)
    mask[rows] = False
    assert np.all(gA.cpu().numpy()[mask] == 0)


@pytest.mark.parametrize("prec", PRECS)
def test_eval_terms(prec, golden):
    g = golden("metrics")
    d = g["A"].shape[1]
    Dp = ops.padded_rank(d)
    idx = g["S_index"]
    out = ops.eval_terms(to_dev(pad(g["A"], Dp)), to_dev(pad(g["B"], Dp)), d,
                         to_dev(idx[0], torch.int32), to_dev(idx[1], torch.int32),
                         to_dev(g["S_value"]), precision=prec).cpu().numpy()
    ref = orc.eval_terms(g["A"], g["B"], idx, g["S_value"])
    np.testing.assert_allclose(out, ref, rtol=SUM_TOL[prec], atol=1e-9)
    np.testing.assert_allclose(orc.metrics_from_terms(out), [g["rmse"], g["jacc"], g["cost"]],
                               rtol=1e-4)


def test_adam_matches_oracle():
    rng = np.random.default_rng(0)
    n = 10007
    p, g = rng.standard_normal(n).astype(np.float32), rng.standard_normal(n).astype(np.float32)
    m, v = np.zeros(n, np.float32), np.zeros(n, np.float32)
    pd, gd, md, vd = (to_dev(x) for x in (p, g, m, v))
    lr, b1, b2, eps = 0.01, 0.9, 0.999, 1e-8
    pr, mr, vr = p.astype(np.float64), m.astype(np.float64), v.astype(np.float64)
    for step in (1, 2, 3):
        ops.adam_step(pd, gd, md, vd, lr / (1 - b1 ** step), 1 / np.sqrt(1 - b2 ** step), b1, b2, eps)
        pr, mr, vr = orc.adam_step(pr, g.astype(np.float64), mr, vr, step, lr, b1, b2, eps)
    np.testing.assert_allclose(pd.cpu().numpy(), pr, rtol=1e-5, atol=1e-6)


def test_bounded_wait_reports_timeout_and_context_survives():
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    ops.wait_flag(flag, 50_000_000)  # 50 ms, nobody sets the flag
    assert _native.read_device_error(0) == 7
    x = torch.ones(4, device="cuda")
    assert float((x * 2).sum().item()) == 8.0


def _relu_bat_c_fp64(A, B, C, chunk=20000):
    """Y = ReLU(B A^T) C in float64 on the device, in row chunks (the oracle's formula)."""
    A64, C64 = A.double(), C.double()
    return torch.cat([torch.relu(B[i:i + chunk].double() @ A64.T) @ C64
                      for i in range(0, B.shape[0], chunk)])


@pytest.mark.parametrize("prec", PRECS)
@pytest.mark.parametrize("D,N,M", [(16, 700, 140000), (32, 500, 80000)])
def test_relu_bat_c_full_tile_groups(D, N, M, prec):
    """Enough row tiles that every CTA holds a full group (8 tiles at d=16, 4 at d=32) and streams
    the chunks once for the whole group: the schedule the C4 workload runs."""
    g = torch.Generator(device="cuda").manual_seed(D + N)
    A = torch.randn(N, D, device="cuda", generator=g)
    B = torch.randn(M, D, device="cuda", generator=g)
    C = torch.randn(N, D, device="cuda", generator=g)
    Y = ops.relu_bat_c(A, B, C, prec)
    _native.raise_device_error(0)
    ref = _relu_bat_c_fp64(A, B, C)
    assert float((Y.double() - ref).abs().max() / ref.abs().max()) < TOL[prec]


@pytest.mark.parametrize("prec", PRECS)
@pytest.mark.parametrize("D,N,M", [(16, 700, 160000), (32, 500, 80000)])
def test_relu_bat_reduce_full_tile_groups(D, N, M, prec):
    g = torch.Generator(device="cuda").manual_seed(D * 7 + N)
    A = torch.randn(M, D, device="cuda", generator=g)
    B = torch.randn(N, D, device="cuda", generator=g)
    out = ops.relu_bat_reduce(A, B, prec)
    _native.raise_device_error(0)
    s1 = s2 = 0.0
    for i in range(0, M, 20000):
        R = torch.relu(A[i:i + 20000].double() @ B.double().T)
        s1 += float(R.sum())
        s2 += float((R * R).sum())
    assert abs(float(out[0]) - s1) / s1 < TOL[prec]
    assert abs(float(out[1]) - s2) / s2 < TOL[prec]


@pytest.mark.parametrize("prec", PRECS)
@pytest.mark.parametrize("k", [10, 20])
def test_relu_bat_c_wide_dynamic_range(prec, k):
    """Rows of R and of C spanning 2^k. TF32 mode runs the second contraction in fp16 with exact
    power-of-two scales (a per-row scale for R from |x_j| max|F_i|, one scale for C from max|C|).
    Here the large rows of F point against every x_j (their S entries are negative and vanish
    under ReLU), so each row of R is carried only by rows of F that are 2^-k smaller than the
    largest, against rows of C that are 2^-k smaller than the largest C row: every output row
    lives 2^-2k below the scales the fp16 operands are normalised to. Checked row by row."""
    rng = np.random.default_rng(100 + k)
    D, Nb, Ns, M = 16, 200, 300, 3000
    u = rng.standard_normal(D)
    u /= np.linalg.norm(u)
    X = (3.0 * u + 0.3 * rng.standard_normal((M, D))) * np.exp2(-rng.uniform(0, k, (M, 1)))
    F_big = -(2.0 * u + 0.1 * rng.standard_normal((Nb, D)))
    F_small = np.exp2(-k) * (u + 0.5 * rng.standard_normal((Ns, D)))
    A = np.vstack([F_big, F_small]).astype(np.float32)
    C = np.vstack([rng.standard_normal((Nb, D)),
                   np.exp2(-k) * rng.standard_normal((Ns, D))]).astype(np.float32)
    X = X.astype(np.float32)
    Y = ops.relu_bat_c(to_dev(A), to_dev(X), to_dev(C), prec).cpu().numpy()
    _native.raise_device_error(0)
    ref = orc.relu_bat_c(A, X, C)
    row_scale = np.abs(ref).max(axis=1)
    assert (row_scale > 0).all()
    row_err = np.abs(Y - ref).max(axis=1) / row_scale
    assert row_err.max() < (1e-3 if prec == ops.SUMAC_TF32 else 1e-5), row_err.max()


@pytest.mark.parametrize("prec", PRECS)
@pytest.mark.parametrize("D", [16, 32, 256])
def test_eval_terms_fnnz_counts_positive_predictions(D, prec):
    """The ninth term of sumac_eval_terms_fnnz: the number of positive entries of A B^T (the
    numerator of fnnz, matlab/sumac/compute_errors.m:62), against a float64 count. Entries whose
    sign the TF32 rounding can flip are counted within a margin."""
    rng = np.random.default_rng(D + 5)
    m, n = 3000, 700
    A = rng.standard_normal((m, D)).astype(np.float32)
    B = rng.standard_normal((n, D)).astype(np.float32)
    keys = rng.choice(m * n, 2000, replace=False)
    ei, ej = (keys // n).astype(np.int32), (keys % n).astype(np.int32)
    v = (0.1 + rng.random(2000)).astype(np.float32)
    Dp = ops.padded_rank(D)
    out = ops.eval_terms(to_dev(pad(A, Dp)), to_dev(pad(B, Dp)), D, to_dev(ei), to_dev(ej),
                         to_dev(v), precision=prec, fnnz=True).cpu().numpy()
    _native.raise_device_error(0)
    L = A.astype(np.float64) @ B.astype(np.float64).T
    exact = int((L > 0).sum())
    scale = np.sqrt(D) * 2e-3 if prec == ops.SUMAC_TF32 else np.sqrt(D) * 1e-6
    ambiguous = int((np.abs(L) < scale).sum())
    assert abs(out[8] - exact) <= ambiguous, (out[8], exact, ambiguous)
    ref = orc.eval_terms(A, B, np.stack([ei, ej]), v)
    np.testing.assert_allclose(out[:8], ref, rtol=SUM_TOL[prec], atol=1e-9)
