"""Metrics (src/sumac/eval.py:111-157) from the eight global terms computed on the device by
``sumac_eval_terms``: rmse = sqrt(ssqe)/|S|, jacc = 1 - num/(sum S + sum Sr - num),
cost = sqrt(errZ)/|S| with ssqe = sum Sr^2 - obs_sq + sum_S (S-ReLU(L))^2 and
errZ = sum Sr^2 - obs_sq + sum_S (S-L)^2."""
from __future__ import annotations

import math

import torch

from . import ops


def metrics_from_terms(t) -> tuple[float, float, float]:
    sum_sr, sum_sr2, obs_sq, res_m, res_l, jnum, sum_v, sum_v2 = (float(x) for x in t)
    s_norm = math.sqrt(sum_v2)
    ssqe = sum_sr2 - obs_sq + res_m
    errz = sum_sr2 - obs_sq + res_l
    rmse = math.sqrt(max(ssqe, 0.0)) / (s_norm + 1e-16)
    jacc = 1.0 - jnum / (sum_v + sum_sr - jnum + 1e-16)
    cost = math.sqrt(max(errz, 0.0)) / (s_norm + 1e-16)
    return rmse, jacc, cost


class Evaluator:
    """Holds the COO support (int32 indices) of the pruned problem on the device. Each call also
    counts the positive entries of A B^T in the same pass: ``fnnz`` is the MATLAB
    implementation's fraction nnz(ReLU(A B^T)) / nnz(S) (matlab/sumac/compute_errors.m:62) of
    the last call."""

    def __init__(self, S_index, S_value, d, precision):
        self.ei = S_index[0].to(torch.int32).contiguous()
        self.ej = S_index[1].to(torch.int32).contiguous()
        self.v = S_value.to(torch.float32).contiguous()
        self.d = d
        self.precision = precision
        self.out = torch.zeros(9, dtype=torch.float64, device=S_value.device)
        self.fnnz = float("nan")

    def __call__(self, Ap, Bp):
        ops.eval_terms(Ap, Bp, self.d, self.ei, self.ej, self.v, self.out, self.precision,
                       fnnz=True)
        t = self.out.cpu().tolist()
        self.fnnz = t[8] / max(self.v.numel(), 1)
        return metrics_from_terms(t[:8])
