"""SALSA solver (src/sumac/training/salsa.py:212-355) driving the native block update.

Per iteration: two reshuffles (one row permutation per factor, drawn from the same seeded
generators as the reference), a device-side rebuild of the per-block CSR of both directions, then
for every block k the update of B against A's row block k followed by the update of A against B's
row block k. Each block update is one ``sumac_salsa_block_update`` call (gather + Gram + LU solve,
the fused tcgen05 product, and the finalize pass with the sparse correction and momentum step).
"""
from __future__ import annotations

import math
import time

import numpy as np
import torch
from torch import Tensor

from . import _native, ops
from .config import SumacConfig
from .data import SparseDirection
from .metrics import Evaluator


def _tall_qr(A: Tensor) -> tuple[Tensor, Tensor] | None:
    """Q, R of a tall, thin float matrix by Cholesky QR in float64: R^T R = A^T A, Q = A R^-1.
    One d x d Gram product and a triangular solve instead of a Householder QR over m rows; in
    float64 its accuracy loss (cond(A)^2 eps64) stays below float32 rounding for cond(A) up to
    ~1e4 and well beyond. None when the Gram matrix is not numerically positive definite."""
    A64 = A.double()
    G = A64.T @ A64
    L, info = torch.linalg.cholesky_ex(G)
    if int(info.item()) != 0:
        return None
    R = L.T
    Q = torch.linalg.solve_triangular(R, A64, upper=True, left=False)
    return Q, R


def refactor(A: Tensor, B: Tensor) -> tuple[Tensor, Tensor]:
    """A B^T unchanged, singular values shared (training/salsa.py:20-33): A = Qa U sqrt(S),
    B = Qb V sqrt(S) from QR factorisations of A and B and the SVD of Ra Rb^T. On the GPU the QRs
    are Cholesky QRs in float64 and the d x d SVD runs on the host: the result does not depend on
    the QR's sign convention (U absorbs it), only, like the reference's, on the SVD's choice of
    signs per singular pair."""
    qa = _tall_qr(A) if A.is_cuda else None
    qb = _tall_qr(B) if qa is not None else None
    if qa is None or qb is None:
        Qa, Ra = torch.linalg.qr(A, mode="reduced")
        Qb, Rb = torch.linalg.qr(B, mode="reduced")
        U, S, Vh = torch.linalg.svd(Ra @ Rb.T, full_matrices=False)
        sqrtS = torch.diag(torch.sqrt(S))
        return Qa @ U @ sqrtS, Qb @ Vh.T @ sqrtS
    (Qa, Ra), (Qb, Rb) = qa, qb
    U, S, Vh = torch.linalg.svd((Ra @ Rb.T).cpu(), full_matrices=False)
    sqrtS = torch.diag(torch.sqrt(S))
    Ua = (U @ sqrtS).to(A.device)
    Vb = (Vh.T @ sqrtS).to(A.device)
    return (Qa @ Ua).to(A.dtype), (Qb @ Vb).to(B.dtype)


def init_salsa_factors(S_index, S_value, m, n, d, gen, dirs=None):
    """A > 0, B < 0 from S times uniform noise, rescaled, then refactored
    (training/salsa.py:36-78); draws from `gen` in the same order as the reference. The uniform
    draws come from `gen` on its own device; the arithmetic runs on the device of S_value. The
    steps (sparse products, closed-form scale, QR + QR + SVD) are the reference's, in its order: the
    same draws in the same order are what makes the initial factors match a reference run.

    On the GPU the sparse products and the scale's sums are native kernels over the entries
    sorted by row and by column (`dirs` = the (A-update, B-update) SparseDirection pair when the
    caller has them, else they are built here); on the CPU it is the reference's torch code."""
    device, dtype = S_value.device, S_value.dtype
    R_A = torch.rand((n, d), device=gen.device, dtype=dtype, generator=gen).to(device)
    R_B = torch.rand((m, d), device=gen.device, dtype=dtype, generator=gen).to(device)
    if device.type == "cuda" and dtype == torch.float32:
        if dirs is None:
            dirs = (SparseDirection(S_index[1], S_index[0], S_value, n, m, 1, csr=False),
                    SparseDirection(S_index[0], S_index[1], S_value, m, n, 1, csr=False))
        dir_a, dir_b = dirs
        A = ops.init_factor(dir_a.out_rowptr(), dir_a.fixed, dir_a.val, R_A, 1.0)
        B = ops.init_factor(dir_b.out_rowptr(), dir_b.fixed, dir_b.val, R_B, -1.0)
        ssqS, SdotL, ssqL = ops.init_scale_terms(A, B, dir_a.out, dir_a.fixed, dir_a.val)
    else:
        with torch.sparse.check_sparse_tensor_invariants(False):
            S = torch.sparse_coo_tensor(S_index.to(device=device, dtype=torch.long), S_value,
                                        size=(m, n), device=device, dtype=dtype).coalesce()
            A = torch.sqrt(torch.sparse.mm(S, R_A))
            B = -torch.sqrt(torch.sparse.mm(S.T, R_B))
        Lij = torch.sum(A[S_index[0], :] * B[S_index[1], :], dim=1)
        ssqS = torch.sum(S_value ** 2)
        ssqL = torch.sum(Lij ** 2)
        SdotL = torch.sum(S_value * Lij)
    a, b, c = ssqL, -2.0 * SdotL, -3.0 * ssqS
    alpha = (-b + torch.sqrt(b ** 2 - 4 * a * c)) / (2 * a)
    scale = torch.clamp(torch.sqrt(alpha), 0.0, 1.0).to(dtype)
    return refactor(scale * A, scale * B)


def make_directions(S_index, S_value, m, n, num_blocks):
    """(A-update, B-update) edge sets: the A-update's fixed rows are the rows of B (columns of S)
    and its updated rows the rows of S; the B-update's the other way round."""
    return (SparseDirection(S_index[1], S_index[0], S_value, n, m, num_blocks),
            SparseDirection(S_index[0], S_index[1], S_value, m, n, num_blocks))


def draw_perm(m: int, gen: torch.Generator, device) -> Tensor:
    """torch.randperm on the generator's device (datasets.py:39), moved to the training device."""
    return torch.randperm(m, device=gen.device, generator=gen).to(device)


def unbias_values(momentum: float, first_step: int, count: int) -> np.ndarray:
    """1 - momentum^step in float32 for steps first_step .. first_step+count-1 (salsa.py:302-303)."""
    mu = np.float32(momentum)
    return np.array([np.float32(1.0) - mu ** np.float32(s)
                     for s in range(first_step, first_step + count)], dtype=np.float32)


# A CUDA graph of the iteration pays off over many iterations only: at C4 the first capture and
# instantiation in a process costs ~0.25 s and a replay saves ~8 % of an eager iteration (62.5
# against 57.7 iterations/s), so eager launches win below ~190 iterations.
GRAPH_MIN_ITERATIONS = 200
# Sharded runs: a rank's eager launches of the exchange and block updates cost more host time
# than its shorter device work, so their graph pays off sooner.
GRAPH_MIN_ITERATIONS_SHARDED = 40


class SalsaState:
    """Device state of one SALSA run: padded factors, momentum, both directions' CSR."""

    def __init__(self, S_index, S_value, m, n, cfg: SumacConfig, A, B, dirs=None):
        dev = cfg.device
        self.d = cfg.rank
        self.Dp = ops.padded_rank(self.d)
        self.m, self.n = m, n
        self.nb = cfg.num_blocks
        self.prec = cfg.precision()
        self.Ap = ops.pad_factor(A.to(torch.float32), self.Dp)
        self.Bp = ops.pad_factor(B.to(torch.float32), self.Dp)
        self.dA = torch.zeros_like(self.Ap)
        self.dB = torch.zeros_like(self.Bp)
        if dirs is None:
            dirs = make_directions(S_index, S_value, m, n, self.nb)
        self.dir_a, self.dir_b = dirs
        self.momentum = float(cfg.momentum)
        self.lrate = float(np.float32(cfg.learning_rate))
        self.unbias = torch.empty(self.nb, dtype=torch.float32, device=dev)
        self.unbias_host = torch.empty(self.nb, dtype=torch.float32).pin_memory() \
            if torch.cuda.is_available() else None
        self.use_graph = True
        self.graph = None
        self.graph_launches = 0      # library kernels captured in the graph
        self.replayed_launches = 0   # library kernels launched by graph replays
        self.eager_done = False
        self.perm_r = torch.empty(m, dtype=torch.int64, device=dev)
        self.perm_c = torch.empty(n, dtype=torch.int64, device=dev)
        L = _native.lib()
        self.ws_b = ops._ws(dev, L.sumac_salsa_update_workspace_bytes(
            n, self.dir_b.block_size, self.d, self.prec), "salsa_b")
        self.ws_a = ops._ws(dev, L.sumac_salsa_update_workspace_bytes(
            m, self.dir_a.block_size, self.d, self.prec), "salsa_a")

    def iteration(self, it: int, perm_r: Tensor, perm_c: Tensor) -> None:
        """One SALSA iteration. The first call runs eagerly; later calls replay a CUDA graph of
        the whole iteration (CSR rebuilds and 2 x num_blocks block updates) that reads the
        permutations and unbias factors from static device buffers."""
        nb = self.nb
        self.unbias_host.copy_(torch.from_numpy(unbias_values(self.momentum, 1 + (it - 1) * nb, nb)))
        self.unbias.copy_(self.unbias_host, non_blocking=True)
        if not self.use_graph:
            self._body(perm_r, perm_c)
            return
        if self.graph is None and self.eager_done:
            self.perm_r.copy_(perm_r)
            self.perm_c.copy_(perm_c)
            g = torch.cuda.CUDAGraph()
            n0 = _native.lib().sumac_kernel_launches()
            with torch.cuda.graph(g):
                self._body(self.perm_r, self.perm_c)
            self.graph_launches = _native.lib().sumac_kernel_launches() - n0
            self.graph = g
            g.replay()
            self.replayed_launches += self.graph_launches
            return
        if self.graph is None:
            self._body(perm_r, perm_c)
            self.eager_done = True
            return
        self.perm_r.copy_(perm_r)
        self.perm_c.copy_(perm_c)
        self.graph.replay()
        self.replayed_launches += self.graph_launches

    def _body(self, perm_r: Tensor, perm_c: Tensor) -> None:
        nb = self.nb
        self.dir_b.rebuild(perm_r)
        self.dir_a.rebuild(perm_c)
        for k in range(nb):
            rows = self.dir_b.block_rows(perm_r, k)
            if rows.numel() > 0:
                ops.salsa_block_update(self.Ap, rows, self.Bp, self.dB, self.d,
                                       self.dir_b.block_rowptr(k), self.dir_b.ent, self.momentum,
                                       self.lrate, self.unbias[k:k + 1], self.prec, self.ws_b)
            rows = self.dir_a.block_rows(perm_c, k)
            if rows.numel() > 0:
                ops.salsa_block_update(self.Bp, rows, self.Ap, self.dA, self.d,
                                       self.dir_a.block_rowptr(k), self.dir_a.ent, self.momentum,
                                       self.lrate, self.unbias[k:k + 1], self.prec, self.ws_a)

    def factors(self):
        return (self.Ap[:, :self.d].contiguous(), self.Bp[:, :self.d].contiguous())


def salsa_loop(S_index: Tensor, S_value: Tensor, m: int, n: int, cfg: SumacConfig,
               A_init: Tensor | None = None, B_init: Tensor | None = None):
    """Same schedule, generators and history as the reference's salsa_loop."""
    assert cfg.num_blocks is not None and cfg.device is not None
    gen, gen_rows, gen_cols = cfg.get_generator()
    dev = cfg.device
    S_index = S_index.to(dev)
    S_value = S_value.to(dev)
    dirs = make_directions(S_index, S_value, m, n, cfg.num_blocks)
    if A_init is None or B_init is None:
        A, B = init_salsa_factors(S_index, S_value, m, n, cfg.rank, gen, dirs=dirs)
    else:
        A, B = A_init.to(dev), B_init.to(dev)
    st = SalsaState(S_index, S_value, m, n, cfg, A, B, dirs=dirs)
    st.use_graph = cfg.max_iterations >= GRAPH_MIN_ITERATIONS
    evaluator = Evaluator(S_index, S_value, cfg.rank, st.prec)
    # the reference's datasets draw one permutation each at construction (datasets.py:34)
    draw_perm(m, gen_rows, dev)
    draw_perm(n, gen_cols, dev)
    rmse, jacc, errZ = evaluator(st.Ap, st.Bp)
    if cfg.verbose:
        print(f"[epoch 0/{cfg.max_iterations}]: cost = {errZ:.6f}, rmse = {rmse:.6f}, "
              f"jacc = {jacc:.6f}, time = 0.0000s")
    hist = {"cost": [], "rmse": [], "jacc": [], "time": []}
    best_cost, best = math.inf, None  # keep_best: the evaluated iterate of lowest cost
    t0 = time.time()
    for it in range(1, cfg.max_iterations + 1):
        perm_r = draw_perm(m, gen_rows, dev)
        perm_c = draw_perm(n, gen_cols, dev)
        st.iteration(it, perm_r, perm_c)
        if cfg.eval_interval is not None and it % cfg.eval_interval == 0:
            rmse, jacc, errZ = evaluator(st.Ap, st.Bp)
            _native.raise_device_error(dev)
            elapsed = time.time() - t0
            hist["cost"].append(errZ)
            hist["rmse"].append(rmse)
            hist["jacc"].append(jacc)
            hist["time"].append(elapsed)
            if cfg.report_fnnz:
                hist.setdefault("fnnz", []).append(evaluator.fnnz)
            if cfg.keep_best and errZ < best_cost:
                best_cost, best = errZ, (st.Ap.clone(), st.Bp.clone())
            if cfg.verbose:
                print(f"[epoch {it}/{cfg.max_iterations}]: cost = {errZ:.6f}, rmse = {rmse:.6f}, "
                      f"jacc = {jacc:.6f}, time = {elapsed:.4f}s")
    _native.raise_device_error(dev)
    if cfg.verbose:
        print(f"\nTotal elapsed time: {time.time() - t0:.2f} sec")
    A, B = st.factors()
    if cfg.keep_best:
        # matlab/sumac/salsa_loop.m:61-79: keep the best evaluated iterate and refactor it
        if best is not None:
            A, B = best[0][:, :st.d].contiguous(), best[1][:, :st.d].contiguous()
        A, B = refactor(A, B)
    return A, B, hist
