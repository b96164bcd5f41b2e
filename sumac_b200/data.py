"""Pre/post-processing (src/sumac/data.py:49-91) and the static sparse structure the solvers read.

``SparseDirection`` holds one update direction of the factorisation on the device: the edges sorted
(stably) by the row of the factor being updated, plus the buffers of the per-block CSR that
``sumac_block_csr_build`` rebuilds after every reshuffle.
"""
from __future__ import annotations

import torch
from torch import Tensor

from . import ops


def prune_zero_rows_cols(S_index: Tensor, shape):
    """Drop all-zero rows / columns and re-index (data.py:49-68). Returns
    (new_index, row_mask, col_mask, m_eff, n_eff); masks are None when nothing is dropped."""
    r, c = S_index
    m, n = shape
    dev = S_index.device
    row_mask = torch.zeros(m, dtype=torch.bool, device=dev)
    row_mask[r] = True
    col_mask = torch.zeros(n, dtype=torch.bool, device=dev)
    col_mask[c] = True
    m_eff = int(row_mask.sum().item())
    n_eff = int(col_mask.sum().item())
    if m_eff == m and n_eff == n:
        return S_index, None, None, m, n
    row_new = torch.full((m,), -1, dtype=torch.long, device=dev)
    row_new[row_mask] = torch.arange(m_eff, device=dev)
    col_new = torch.full((n,), -1, dtype=torch.long, device=dev)
    col_new[col_mask] = torch.arange(n_eff, device=dev)
    return torch.stack([row_new[r], col_new[c]]), row_mask, col_mask, m_eff, n_eff


def restore_zero_rows_cols(A, B, m, n, rank, row_mask, col_mask):
    """Scatter the factors back to the original shape, zeros for dropped rows (data.py:71-91)."""
    if row_mask is not None:
        A_ori = torch.zeros((m, rank), dtype=A.dtype, device=A.device)
        A_ori[row_mask] = A
    else:
        A_ori = A
    if col_mask is not None:
        B_ori = torch.zeros((n, rank), dtype=B.dtype, device=B.device)
        B_ori[col_mask] = B
    else:
        B_ori = B
    return A_ori, B_ori


class SparseDirection:
    """Edges of S for one update direction: ``fixed`` indexes the rows of the fixed factor,
    ``out`` the rows of the updated factor (M of them), sorted stably by ``out``."""

    def __init__(self, fixed: Tensor, out: Tensor, val: Tensor, m_fixed: int, M: int,
                 num_blocks: int, csr: bool = True):
        # a stable radix sort of 32-bit keys (half the passes of int64 keys)
        out_sorted, order = torch.sort(out.to(torch.int32), stable=True)
        self.out = out_sorted.contiguous()
        self.fixed = fixed.to(torch.int32)[order].contiguous()
        self.val = val[order].to(torch.float32).contiguous()
        self.m_fixed = int(m_fixed)
        self.M = int(M)
        self.nnz = int(val.numel())
        self.num_blocks = int(num_blocks)
        self.block_size = (self.m_fixed + num_blocks - 1) // num_blocks
        dev = val.device
        self._out_rowptr = None
        if csr:  # per-block CSR storage (rebuild)
            self.rowptr = torch.empty(num_blocks * self.M + 1, dtype=torch.int32, device=dev)
            self.ent = torch.empty((max(self.nnz, 1), 2), dtype=torch.int32, device=dev)

    def out_rowptr(self) -> Tensor:
        """[M + 1] int32: the entries of updated row r are [rowptr[r], rowptr[r + 1])."""
        if self._out_rowptr is None:
            q = torch.arange(self.M + 1, dtype=torch.int32, device=self.out.device)
            self._out_rowptr = torch.searchsorted(self.out, q).to(torch.int32)
        return self._out_rowptr

    def rebuild(self, perm: Tensor) -> None:
        """Per-block CSR for the row permutation ``perm`` of the fixed factor."""
        ops.block_csr_build(perm, self.num_blocks, self.fixed, self.out, self.val, self.M,
                            self.rowptr, self.ent)

    def block_rows(self, perm: Tensor, k: int) -> Tensor:
        bs = self.block_size
        return perm[k * bs:min(self.m_fixed, (k + 1) * bs)]

    def block_rowptr(self, k: int) -> Tensor:
        return self.rowptr[k * self.M:(k + 1) * self.M + 1]
