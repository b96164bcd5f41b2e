"""CPU oracle for the sumac hot path. TEST INFRASTRUCTURE ONLY.

This module restates, in numpy float64, the algorithm of flatironinstitute/sumac on the path that
sumac_b200 accelerates on the GPU. Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s
``cpu_baseline`` / ``--impl reference`` legs may import it, and only as the checker or as the timed
CPU baseline. The product path (``sumac_b200``) never imports it and has no CPU fallback.

Pinning: every function here is checked against golden vectors produced by running the reference's
own Python code (``tests/golden/make_golden.py`` writes ``tests/golden/*.npz``; the checks are in
``tests/test_oracle_golden.py``).

Citations are ``path:line`` inside the reference project (flatironinstitute/sumac).
"""
from __future__ import annotations

import math
import numpy as np

F64 = np.float64


def relu(x):
    return np.maximum(x, 0.0)


# --------------------------------------------------------------------------------------------
# Kernels (dense, unmasked): relu_bat_c and relu_bat_reduce
# --------------------------------------------------------------------------------------------

def relu_bat_c(A, B, C):
    """Y = ReLU(B @ A.T) @ C  (src/sumac/kernels/tuning/relu_bat_c/relu_bat_c_base.py:4-6)."""
    A, B, C = (np.asarray(x, F64) for x in (A, B, C))
    return relu(B @ A.T) @ C


def relu_bat_reduce(A, B):
    """(sum ReLU(A B^T), sum ReLU(A B^T)^2) in float64
    (src/sumac/kernels/tuning/relu_bat_reduce/relu_bat_reduce.py:11-22)."""
    A, B = np.asarray(A, F64), np.asarray(B, F64)
    sr = relu(A @ B.T)
    return float(sr.sum()), float((sr * sr).sum())


# --------------------------------------------------------------------------------------------
# Masked residual and the SALSA least-squares block step
# --------------------------------------------------------------------------------------------

def masked_residual(A_I, B, edge_i, edge_j, vals):
    """R[j, i] = ReLU(L[j, i]) off the support, L[j, i] - S[i, j] on it, with L = B @ A_I^T.

    Off-support entries penalise only positive predictions; on-support entries use the raw
    residual L - S (salsa.py:98-115 via lsqB = B - ReLU(L) P + (S - L + ReLU(L)) P;
    kernels/relu_batc_jit/kernel_fused.cu:117-133).
    """
    L = np.asarray(B, F64) @ np.asarray(A_I, F64).T
    R = relu(L)
    ei = np.asarray(edge_i, np.int64)
    ej = np.asarray(edge_j, np.int64)
    R[ej, ei] = L[ej, ei] - np.asarray(vals, F64)
    return R


def pinv_t(A_I):
    """P = solve(A_I^T A_I, A_I^T)^T   (training/salsa.py:138-140)."""
    A_I = np.asarray(A_I, F64)
    G = A_I.T @ A_I
    return np.linalg.solve(G, A_I.T).T


def lsq_update(A_I, B, P, dB, edge_i, edge_j, vals, momentum, unbias, lrate):
    """One SALSA least-squares update of the factor B against the fixed block A_I.

    Follows training/salsa.py:84-116 term by term:
      stepM = ReLU(B A_I^T) P;  L_ij = <A_I[i], B[j]>;  Ct = v - L + ReLU(L)
      stepC[j] += Ct * P[i];    lsqB = B - stepM + stepC
      dB' = (lsqB - B)(1 - mu) + dB mu;  B' = B + lr dB' / unbias
    """
    A_I, B, P, dB = (np.asarray(x, F64) for x in (A_I, B, P, dB))
    ei = np.asarray(edge_i, np.int64)
    ej = np.asarray(edge_j, np.int64)
    v = np.asarray(vals, F64)
    stepM = relu(B @ A_I.T) @ P
    Lij = np.sum(A_I[ei] * B[ej], axis=1)
    Ct = v - Lij + relu(Lij)
    stepC = np.zeros_like(B)
    np.add.at(stepC, ej, Ct[:, None] * P[ei])
    lsqB = B - stepM + stepC
    dB_new = (lsqB - B) * (1.0 - momentum) + dB * momentum
    B_new = B + lrate * dB_new / unbias
    return B_new, dB_new


def block_update(F_fixed, row_indices, B, dB, S_index, S_value, edge_idx, momentum, unbias, lrate):
    """SALSA update of B against the rows ``row_indices`` of the fixed factor
    (training/salsa.py:119-166): gather, Gram solve, local re-index, lsq_update."""
    F_fixed = np.asarray(F_fixed, F64)
    rows = np.asarray(row_indices, np.int64)
    A_I = F_fixed[rows]
    P = pinv_t(A_I)
    S_index = np.asarray(S_index, np.int64)
    eidx = np.asarray(edge_idx, np.int64)
    local_map = np.zeros(F_fixed.shape[0], np.int64)
    local_map[rows] = np.arange(rows.size)
    edge_i = local_map[S_index[0, eidx]]
    edge_j = S_index[1, eidx]
    return lsq_update(A_I, B, P, dB, edge_i, edge_j, np.asarray(S_value, F64)[eidx],
                      momentum, unbias, lrate)


# --------------------------------------------------------------------------------------------
# Row-block partition (StochasticRowBlockDataset) and the per-block CSR it implies
# --------------------------------------------------------------------------------------------

def block_partition(perm, edge_rows, num_blocks):
    """Given perm (a permutation of the m fixed rows) return (block_size, block_of_edge,
    local_index_of_edge, row lists), following datasets.py:37-58: perm_inv[perm] = arange,
    block_size = ceil(m / nb), edge block = perm_inv[row] // block_size, block k's rows are
    perm[k*bs : (k+1)*bs] and an edge's local row index is its position in that list
    (salsa.py:145-148)."""
    perm = np.asarray(perm, np.int64)
    m = perm.size
    perm_inv = np.empty_like(perm)
    perm_inv[perm] = np.arange(m)
    bs = (m + num_blocks - 1) // num_blocks
    pos = perm_inv[np.asarray(edge_rows, np.int64)]
    blk = pos // bs
    local = pos - blk * bs
    rows = [perm[k * bs:min(m, (k + 1) * bs)] for k in range(num_blocks)]
    return bs, blk, local, rows


def block_edge_sets(perm, edge_rows, num_blocks):
    """Per block, the sorted array of edge ids in it (the set the reference's
    ``block_edge_idx[k]`` holds, datasets.py:45-58; argsort is unstable so only the set is
    defined)."""
    _, blk, _, _ = block_partition(perm, edge_rows, num_blocks)
    return [np.sort(np.nonzero(blk == k)[0]) for k in range(num_blocks)]


def block_csr(perm, fixed_rows, out_rows, vals, num_blocks, M):
    """Canonical per-block CSR keyed by (block, output row): rowptr[k*M + j] is the first entry
    of output row j in block k; entries carry (local fixed index, value). Within one key the
    entries keep the order of the input edge list after a stable sort by output row, which is
    the order the GPU builder produces (bit-exact contract)."""
    fixed_rows = np.asarray(fixed_rows, np.int64)
    out_rows = np.asarray(out_rows, np.int64)
    vals = np.asarray(vals, np.float32)
    order = np.argsort(out_rows, kind="stable")
    _, blk, local, _ = block_partition(perm, fixed_rows[order], num_blocks)
    key = blk * M + out_rows[order]
    o2 = np.argsort(key, kind="stable")
    key_sorted = key[o2]
    rowptr = np.searchsorted(key_sorted, np.arange(num_blocks * M + 1), side="left").astype(np.int64)
    return rowptr, local[o2].astype(np.int32), vals[order][o2]


# --------------------------------------------------------------------------------------------
# Loss / metrics (eval.py) and the GD block gradient
# --------------------------------------------------------------------------------------------

def block_loss_terms(A_I, B, local_r, cols, vals):
    """Per-block terms of eval.py:14-38 (block_loss_errz) with the dense sums of relu_bat_reduce:
    returns (mse_full, sum_sr, jacc_num, errZ_num) in float64."""
    A_I, B = np.asarray(A_I, F64), np.asarray(B, F64)
    sum_sr, sum_sr2 = relu_bat_reduce(A_I, B)
    v = np.asarray(vals, F64)
    L = np.sum(A_I[np.asarray(local_r)] * B[np.asarray(cols)], axis=1)
    M = relu(L)
    obs_sq = float((M * M).sum())
    mse_full = sum_sr2 - obs_sq + float(((v - M) ** 2).sum())
    errZ = sum_sr2 - obs_sq + float(((v - L) ** 2).sum())
    jacc = float(np.minimum(v, M).sum())
    return mse_full, sum_sr, jacc, errZ


def metrics_from_terms(t):
    """(rmse, jacc, cost) from the eight global terms {sum ReLU(L), sum ReLU(L)^2,
    sum_S ReLU(L)^2, sum_S (S-ReLU(L))^2, sum_S (S-L)^2, sum_S min(S,ReLU(L)), sum S, sum S^2}
    (eval.py:150-157)."""
    sum_sr, sum_sr2, obs_sq, res_m, res_l, jnum, sum_v, sum_v2 = (float(x) for x in t)
    S_norm = math.sqrt(sum_v2)
    ssqe = sum_sr2 - obs_sq + res_m
    errZ = sum_sr2 - obs_sq + res_l
    rmse = math.sqrt(max(ssqe, 0.0)) / (S_norm + 1e-16)
    jacc = 1.0 - jnum / (sum_v + sum_sr - jnum + 1e-16)
    cost = math.sqrt(max(errZ, 0.0)) / (S_norm + 1e-16)
    return rmse, jacc, cost


def eval_terms(A, B, S_index, S_value):
    """The eight global terms of metrics_from_terms, in float64."""
    A, B = np.asarray(A, F64), np.asarray(B, F64)
    idx = np.asarray(S_index, np.int64)
    v = np.asarray(S_value, F64)
    s1, s2 = relu_bat_reduce(A, B)
    L = np.sum(A[idx[0]] * B[idx[1]], axis=1)
    M = relu(L)
    return np.array([s1, s2, (M * M).sum(), ((v - M) ** 2).sum(), ((v - L) ** 2).sum(),
                     np.minimum(v, M).sum(), v.sum(), (v * v).sum()])


def evaluate(A, B, S_index, S_value, block_rows):
    """Global metrics (eval.py:111-157): returns (rmse, jacc, cost) where cost = sqrt(errZ)/|S|.
    ``block_rows`` is the list of row blocks; the result does not depend on the partition except
    through summation order."""
    A, B = np.asarray(A, F64), np.asarray(B, F64)
    S_index = np.asarray(S_index, np.int64)
    v = np.asarray(S_value, F64)
    ssqe = sumSr = num_j = errZ = 0.0
    row_of = S_index[0]
    for rows in block_rows:
        rows = np.asarray(rows, np.int64)
        local = np.full(A.shape[0], -1, np.int64)
        local[rows] = np.arange(rows.size)
        sel = np.nonzero(local[row_of] >= 0)[0]
        a, b, c, d = block_loss_terms(A[rows], B, local[row_of[sel]], S_index[1, sel], v[sel])
        ssqe += a; sumSr += b; num_j += c; errZ += d
    S_norm = float(np.linalg.norm(v))
    rmse = math.sqrt(ssqe) / (S_norm + 1e-16)
    denom = v.sum() + sumSr - num_j
    jacc = 1.0 - num_j / (denom + 1e-16)
    cost = math.sqrt(errZ) / (S_norm + 1e-16)
    return rmse, jacc, cost


def gd_block_grad(A_I, B, local_r, cols, vals):
    """errZ of one row block and its gradients (eval.py:24-34 through autograd and
    kernels/relu_bat_reduce_jit/custom_op.py:39-85): dLoss/dL = 2R with R the masked residual
    (ReLU(L) off the support, L - S on it), so grad_A_I = 2 R B and grad_B = 2 R^T A_I
    (here R is b x n, L = A_I B^T)."""
    A_I, B = np.asarray(A_I, F64), np.asarray(B, F64)
    L = A_I @ B.T
    R = relu(L)
    lr_ = np.asarray(local_r, np.int64)
    cc = np.asarray(cols, np.int64)
    v = np.asarray(vals, F64)
    Lo = L[lr_, cc]
    errZ = float((R * R).sum() - (relu(Lo) ** 2).sum() + ((v - Lo) ** 2).sum())
    R[lr_, cc] = Lo - v
    return errZ, 2.0 * R @ B, 2.0 * R.T @ A_I


def adam_step(p, g, m, v, step, lr, beta1, beta2, eps):
    """torch.optim.Adam (weight_decay=0, no amsgrad) single-tensor update, as sumac's GD uses it
    (training/gd.py:20-30): m = lerp(m, g, 1-b1); v = b2 v + (1-b2) g^2;
    p -= lr/(1-b1^t) * m / (sqrt(v)/sqrt(1-b2^t) + eps)."""
    m = m + (g - m) * (1.0 - beta1)
    v = v * beta2 + (1.0 - beta2) * g * g
    bc1 = 1.0 - beta1 ** step
    bc2 = 1.0 - beta2 ** step
    denom = np.sqrt(v) / math.sqrt(bc2) + eps
    p = p - (lr / bc1) * m / denom
    return p, m, v


# --------------------------------------------------------------------------------------------
# End-to-end loops with injected permutations (small sizes only)
# --------------------------------------------------------------------------------------------

def salsa_iterations(S_index, S_value, m, n, A, B, num_blocks, iters, momentum, lrate,
                     perms_rows, perms_cols):
    """salsa_loop's update schedule (training/salsa.py:290-313) with the per-iteration
    permutations supplied: for block k, update B against A's row block k, then A against B's
    row block k (the transposed problem). Momentum buffers start at zero; the unbias step
    counter is mb + 1 + (iter-1) nb (salsa.py:302-303). Returns A, B (float64)."""
    S_index = np.asarray(S_index, np.int64)
    S_T = S_index[[1, 0]]
    A = np.asarray(A, F64).copy(); B = np.asarray(B, F64).copy()
    dA = np.zeros_like(A); dB = np.zeros_like(B)
    mu = np.float32(momentum)
    for it in range(1, iters + 1):
        prow, pcol = perms_rows[it - 1], perms_cols[it - 1]
        sets_r = block_edge_sets(prow, S_index[0], num_blocks)
        sets_c = block_edge_sets(pcol, S_T[0], num_blocks)
        _, _, _, rows_r = block_partition(prow, S_index[0], num_blocks)
        _, _, _, rows_c = block_partition(pcol, S_T[0], num_blocks)
        for k in range(num_blocks):
            step = k + 1 + (it - 1) * num_blocks
            unbias = float(np.float32(1.0) - mu ** np.float32(step))
            B, dB = block_update(A, rows_r[k], B, dB, S_index, S_value, sets_r[k],
                                 float(mu), unbias, lrate)
            A, dA = block_update(B, rows_c[k], A, dA, S_T, S_value, sets_c[k],
                                 float(mu), unbias, lrate)
    return A, B


def gd_epochs(S_index, S_value, A, B, block_rows, batches, epochs, lr, betas=(0.9, 0.999),
              eps=1e-8):
    """GD_loop's training schedule (training/gd.py:173-200) with Adam: for each batch of blocks,
    sum the block losses, take gradients w.r.t. all of A and B, one Adam step over both full
    factors. ``batches`` is the list (per epoch) of lists of block ids."""
    S_index = np.asarray(S_index, np.int64)
    v = np.asarray(S_value, F64)
    A = np.asarray(A, F64).copy(); B = np.asarray(B, F64).copy()
    mA = np.zeros_like(A); vA = np.zeros_like(A)
    mB = np.zeros_like(B); vB = np.zeros_like(B)
    step = 0
    for ep in range(epochs):
        for batch in batches[ep]:
            gA = np.zeros_like(A); gB = np.zeros_like(B)
            for k in batch:
                rows = np.asarray(block_rows[k], np.int64)
                local = np.full(A.shape[0], -1, np.int64)
                local[rows] = np.arange(rows.size)
                sel = np.nonzero(local[S_index[0]] >= 0)[0]
                _, ga, gb = gd_block_grad(A[rows], B, local[S_index[0, sel]], S_index[1, sel], v[sel])
                gA[rows] += ga
                gB += gb
            step += 1
            A, mA, vA = adam_step(A, gA, mA, vA, step, lr, betas[0], betas[1], eps)
            B, mB, vB = adam_step(B, gB, mB, vB, step, lr, betas[0], betas[1], eps)
    return A, B
