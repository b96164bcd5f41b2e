"""Torch-facing operations over the C ABI (include/sumac_b200.h).

Each function checks its tensors, sizes a workspace through the matching ``*_workspace_bytes``
query, and enqueues the native kernels on the current CUDA stream. Errors from the C layer become
``ValueError`` (bad arguments), ``NotImplementedError`` (rank / precision not built) or
``RuntimeError``. Every function requires CUDA tensors; there is no CPU path.
"""
from __future__ import annotations

import torch

from . import _native as N
from ._native import SUMAC_3XTF32, SUMAC_TF32, check, ptr


def precision_code(allow_tf32: bool) -> int:
    """allow_tf32=True -> one TF32 pass; False -> 3xTF32 (fp32-accurate, the reference default)."""
    return SUMAC_TF32 if allow_tf32 else SUMAC_3XTF32


def padded_rank(d: int) -> int:
    dp = N.lib().sumac_padded_rank(int(d))
    if dp <= 0:
        raise NotImplementedError(f"rank {d} is not supported (max 256)")
    return dp


def _cuda_f32(name, t, ndim=2):
    if not isinstance(t, torch.Tensor) or t.device.type != "cuda":
        raise ValueError(f"{name} must be a CUDA tensor")
    if t.dtype != torch.float32:
        raise ValueError(f"{name} must be float32, got {t.dtype}")
    if t.dim() != ndim:
        raise ValueError(f"{name} must be {ndim}-D, got shape {tuple(t.shape)}")
    return t.contiguous()


def _ws(device, nbytes, tag="main"):
    return N.workspace(device, nbytes, tag)


def pad_factor(F: torch.Tensor, Dp: int | None = None) -> torch.Tensor:
    """Copy a [rows, d] factor into a zero-padded [rows, Dp] contiguous fp32 tensor."""
    d = F.shape[1]
    Dp = Dp or padded_rank(d)
    out = torch.zeros((F.shape[0], Dp), dtype=torch.float32, device=F.device)
    out[:, :d] = F
    return out


# ------------------------------------------------------------------ reference ops
SUMAC_RELU, SUMAC_STEP = 0, 1


def relu_bat_c(A, B, C, precision=SUMAC_3XTF32, mode=SUMAC_RELU):
    """Y = ReLU(B A^T) C with A[N, D], B[M, D], C[N, D] (relu_bat_c_base.py:4-6); with
    mode=SUMAC_STEP, Y = step(B A^T) C (1 where B A^T > 0, else 0)."""
    A, B, C = _cuda_f32("A", A), _cuda_f32("B", B), _cuda_f32("C", C)
    Nr, D = A.shape
    M, DB = B.shape
    if DB != D or tuple(C.shape) != (Nr, D):
        raise ValueError("shape mismatch")
    Y = torch.empty((M, D), dtype=torch.float32, device=A.device)
    if M == 0:
        return Y
    if Nr == 0:
        return Y.zero_()
    L = N.lib()
    nb = L.sumac_relu_bat_c_workspace_bytes(M, Nr, D, precision)
    if nb == 0:
        raise NotImplementedError(f"relu_bat_c: D={D} not supported")
    ws = _ws(A.device, nb)
    check(L.sumac_relu_bat_c_mode(ptr(A), ptr(B), ptr(C), M, Nr, D, ptr(Y), precision, int(mode),
                                  ptr(ws), ws.numel(), ptr(N.err_word(A.device)),
                                  N.stream_ptr(A.device)), "relu_bat_c")
    return Y


def relu_bat_reduce(A, B, precision=SUMAC_3XTF32):
    """(sum ReLU(A B^T), sum ReLU(A B^T)^2) as a float64 tensor [2] on the device."""
    A, B = _cuda_f32("A", A), _cuda_f32("B", B)
    M, D = A.shape
    Nr, DB = B.shape
    if DB != D:
        raise ValueError("shape mismatch")
    out = torch.zeros(2, dtype=torch.float64, device=A.device)
    if M == 0 or Nr == 0:
        return out
    L = N.lib()
    nb = L.sumac_relu_bat_reduce_workspace_bytes(M, Nr, D, precision)
    if nb == 0:
        raise NotImplementedError(f"relu_bat_reduce: D={D} not supported")
    ws = _ws(A.device, nb)
    check(L.sumac_relu_bat_reduce(ptr(A), ptr(B), M, Nr, D, ptr(out), precision, ptr(ws),
                                  ws.numel(), ptr(N.err_word(A.device)), N.stream_ptr(A.device)),
          "relu_bat_reduce")
    return out


# ------------------------------------------------------------------ masked product
def masked_product(X, F, C, rowptr=None, ent=None, precision=SUMAC_3XTF32):
    """Y = R C with R = ReLU(X F^T) off the support and X F^T - S on it (padded operands)."""
    X, F, C = _cuda_f32("X", X), _cuda_f32("F", F), _cuda_f32("C", C)
    M, Dp = X.shape
    Nr = F.shape[0]
    Y = torch.empty((M, Dp), dtype=torch.float32, device=X.device)
    L = N.lib()
    ws = _ws(X.device, L.sumac_masked_product_workspace_bytes(M, Nr, Dp, precision))
    check(L.sumac_masked_product(ptr(X), ptr(F), ptr(C), M, Nr, Dp, ptr(rowptr), ptr(ent), ptr(Y),
                                 precision, ptr(ws), ws.numel(), ptr(N.err_word(X.device)),
                                 N.stream_ptr(X.device)), "masked_product")
    return Y


# ------------------------------------------------------------------ CSR
def block_csr_build(perm, num_blocks, e_fixed, e_out, e_val, M, rowptr=None, ent=None):
    """Per-block CSR after a reshuffle. perm: int64 permutation of the fixed rows; e_*: edges
    sorted (stably) by output row. Returns (rowptr[int32, nb*M+1], ent[int32, nnz, 2])."""
    dev = perm.device
    m_fixed = perm.numel()
    nnz = e_fixed.numel()
    if rowptr is None:
        rowptr = torch.empty(num_blocks * M + 1, dtype=torch.int32, device=dev)
    if ent is None:
        ent = torch.empty((max(nnz, 1), 2), dtype=torch.int32, device=dev)
    L = N.lib()
    ws = _ws(dev, L.sumac_block_csr_workspace_bytes(m_fixed, nnz, num_blocks, M), "csr")
    check(L.sumac_block_csr_build(ptr(perm), m_fixed, num_blocks, ptr(e_fixed), ptr(e_out),
                                  ptr(e_val), nnz, M, ptr(rowptr), ptr(ent), ptr(ws), ws.numel(),
                                  N.stream_ptr(dev)), "block_csr_build")
    return rowptr, ent


# ------------------------------------------------------------------ SALSA
def salsa_block_update(F, rows, X, dX, d, rowptr, ent, momentum, lrate, unbias,
                       precision=SUMAC_3XTF32, ws=None):
    """In-place SALSA update of padded X / dX against rows `rows` of padded F."""
    L = N.lib()
    dev = X.device
    b = rows.numel()
    M = X.shape[0]
    if ws is None:
        ws = _ws(dev, L.sumac_salsa_update_workspace_bytes(M, b, d, precision), "salsa")
    check(L.sumac_salsa_block_update(ptr(F), F.shape[0], ptr(rows), b, ptr(X), ptr(dX), M, d,
                                     ptr(rowptr), ptr(ent), float(momentum), float(lrate),
                                     ptr(unbias), precision, ptr(ws), ws.numel(),
                                     ptr(N.err_word(dev)), N.stream_ptr(dev)),
          "salsa_block_update")


# ------------------------------------------------------------------ GD
def gd_block_grad(A, B, d, rows, rowptr_b, ent_b, rowptr_a, ent_a, gA, gB, accumulate,
                  precision=SUMAC_3XTF32):
    L = N.lib()
    dev = A.device
    n, b = B.shape[0], rows.numel()
    ws = _ws(dev, L.sumac_gd_grad_workspace_bytes(n, b, d, precision), "gd")
    check(L.sumac_gd_block_grad(ptr(A), ptr(B), n, d, ptr(rows), b, ptr(rowptr_b), ptr(ent_b),
                                ptr(rowptr_a), ptr(ent_a), ptr(gA), ptr(gB), int(accumulate),
                                precision, ptr(ws), ws.numel(), ptr(N.err_word(dev)),
                                N.stream_ptr(dev)), "gd_block_grad")


def eval_terms(A, B, d, ei, ej, v, out=None, precision=SUMAC_3XTF32, fnnz=False):
    """Eight float64 metric terms (see include/sumac_b200.h) on the device; with fnnz=True a
    ninth, the number of positive entries of A B^T."""
    L = N.lib()
    dev = A.device
    m, n, nnz = A.shape[0], B.shape[0], v.numel()
    if out is None:
        out = torch.zeros(9 if fnnz else 8, dtype=torch.float64, device=dev)
    ws = _ws(dev, L.sumac_eval_terms_workspace_bytes(m, n, nnz, d, precision), "eval")
    fn = L.sumac_eval_terms_fnnz if fnnz else L.sumac_eval_terms
    check(fn(ptr(A), ptr(B), m, n, d, ptr(ei), ptr(ej), ptr(v), nnz, ptr(out), precision, ptr(ws),
             ws.numel(), ptr(N.err_word(dev)), N.stream_ptr(dev)), "eval_terms")
    return out


def block_loss_terms(A, B, d, rows, rowptr_b, ent_b, out, accumulate, precision=SUMAC_3XTF32):
    L = N.lib()
    dev = A.device
    n, b = B.shape[0], rows.numel()
    ws = _ws(dev, L.sumac_block_loss_workspace_bytes(n, b, d, precision), "loss")
    check(L.sumac_block_loss_terms(ptr(A), ptr(B), n, d, ptr(rows), b, ptr(rowptr_b), ptr(ent_b),
                                   ptr(out), int(accumulate), precision, ptr(ws), ws.numel(),
                                   ptr(N.err_word(dev)), N.stream_ptr(dev)), "block_loss_terms")
    return out


def adam_step(p, g, m, v, lr_over_bc1, inv_sqrt_bc2, beta1, beta2, eps):
    check(N.lib().sumac_adam_step(ptr(p), ptr(g), ptr(m), ptr(v), p.numel(), float(lr_over_bc1),
                                  float(inv_sqrt_bc2), float(beta1), float(beta2), float(eps),
                                  N.stream_ptr(p.device)), "adam_step")


def grad_sumsq(g, out):
    check(N.lib().sumac_grad_sumsq(ptr(g), g.numel(), ptr(out), N.stream_ptr(g.device)), "grad_sumsq")


def sgd_step(p, g, buf, lr, momentum, first, sumsq, max_norm):
    check(N.lib().sumac_sgd_step(ptr(p), ptr(g), ptr(buf), p.numel(), float(lr), float(momentum),
                                 int(first), ptr(sumsq), float(max_norm), N.stream_ptr(p.device)),
          "sgd_step")


def fill_zero(t):
    check(N.lib().sumac_fill_zero(ptr(t), t.numel(), N.stream_ptr(t.device)), "fill_zero")


def wait_flag(flag, timeout_ns):
    dev = flag.device
    check(N.lib().sumac_wait_flag(ptr(flag), ptr(N.err_word(dev)), int(timeout_ns),
                                  N.stream_ptr(dev)), "wait_flag")


def gather_owned_rows(local, lo, hi, rows, out):
    """out[p] = F[rows[p]] for the rows [lo, hi) this rank holds as `local`, zero elsewhere."""
    L = N.lib()
    check(L.sumac_gather_owned_rows(ptr(local), int(lo), int(hi), ptr(rows), rows.numel(),
                                    local.shape[1], ptr(out), N.stream_ptr(out.device)),
          "gather_owned_rows")


def init_factor(rowptr, col, val, R, sign):
    """sign * sqrt(S R) row by row, S given by its row-sorted entries (rowptr[M+1], col, val)
    (the sparse products of init_salsa_factors, training/salsa.py:46-50)."""
    R = _cuda_f32("R", R)
    M, d = rowptr.numel() - 1, R.shape[1]
    out = torch.empty((M, d), dtype=torch.float32, device=R.device)
    check(N.lib().sumac_init_factor(ptr(rowptr), ptr(col), ptr(val), M, ptr(R), d, float(sign),
                                    ptr(out), N.stream_ptr(R.device)), "init_factor")
    return out


def init_scale_terms(A, B, ei, ej, v):
    """float64 device tensor (sum v^2, sum v L, sum L^2), L = <A[ei], B[ej]> per entry (the sums
    of the closed-form scale of init_salsa_factors, training/salsa.py:52-59)."""
    A, B = _cuda_f32("A", A), _cuda_f32("B", B)
    L = N.lib()
    out = torch.empty(3, dtype=torch.float64, device=A.device)
    nb = L.sumac_init_scale_workspace_bytes()
    ws = _ws(A.device, nb, "init_scale")
    check(L.sumac_init_scale_terms(ptr(A), ptr(B), A.shape[1], ptr(ei), ptr(ej), ptr(v), v.numel(),
                                   ptr(out), ptr(ws), nb, N.stream_ptr(A.device)), "init_scale_terms")
    return out


def assemble_rows_p2p(local, lo, hi, rows, nrows, slot_floats, peer_bufs, peer_flags, epoch,
                      rank, world):
    """Row exchange over NVLink peer memory (sumac_assemble_rows_p2p): this rank's rows of
    rows[:nrows] into slot (epoch + 1) & 1 of every rank's buffer, then a flag barrier."""
    dev = epoch.device
    check(N.lib().sumac_assemble_rows_p2p(ptr(local), int(lo), int(hi), ptr(rows), int(nrows),
                                          local.shape[1], int(slot_floats), ptr(peer_bufs),
                                          ptr(peer_flags), ptr(epoch), int(rank), int(world),
                                          ptr(N.err_word(dev)), N.stream_ptr(dev)),
          "assemble_rows_p2p")
