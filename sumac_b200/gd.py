"""GD solver (src/sumac/training/gd.py:110-253) driving the native block gradient and optimizer.

Per batch of row blocks: the loss terms (report epochs only, before the step, as the reference
computes its loss in the forward pass), the block gradients ``sumac_gd_block_grad`` (two fused
tcgen05 passes, no b x n intermediate), then one optimizer step over both full factors
(Adam/AdamW/SGD natively; Muon through torch.optim.Muon on the unpadded views).
"""
from __future__ import annotations

import math
import time

import torch
from torch import Tensor
from torch.utils.data import DataLoader

from . import _native, ops
from .config import OptimizerName, SumacConfig
from .data import SparseDirection
from .metrics import Evaluator, metrics_from_terms
from .salsa import draw_perm, init_salsa_factors


class _Optimizer:
    """torch.optim semantics over the padded factors (training/gd.py:20-46)."""

    def __init__(self, cfg: SumacConfig, params: list[Tensor], grads: list[Tensor], d: int,
                 sum_group=None):
        """sum_group: the last param / grad is this rank's slice of a factor sharded over the
        group (the others are replicated): SGD's clipping norm adds the slices' squared norms
        over the group."""
        self.sum_group = sum_group
        self.cfg = cfg
        self.params = params
        self.grads = grads
        self.kind = cfg.optimizer
        self.step_count = 0
        if self.kind in (OptimizerName.ADAM, OptimizerName.ADAMW):
            self.m = [torch.zeros_like(p) for p in params]
            self.v = [torch.zeros_like(p) for p in params]
        elif self.kind == OptimizerName.SGD:
            self.buf = [torch.zeros_like(p) for p in params]
            self.sumsq = torch.zeros(1, dtype=torch.float64, device=params[0].device)
        elif self.kind == OptimizerName.MUON:
            self.views = [torch.nn.Parameter(p[:, :d]) for p in params]
            self.torch_opt = torch.optim.Muon(self.views, lr=cfg.learning_rate, weight_decay=0.0,
                                              momentum=cfg.momentum,
                                              adjust_lr_fn="match_rms_adamw")
        else:
            raise ValueError(f"Unknown optimizer: {cfg.optimizer}")

    def step(self) -> None:
        self.step_count += 1
        t = self.step_count
        cfg = self.cfg
        if self.kind in (OptimizerName.ADAM, OptimizerName.ADAMW):
            b1, b2 = cfg.adam_betas
            lr_bc1 = cfg.learning_rate / (1.0 - b1 ** t)
            inv_sqrt_bc2 = 1.0 / math.sqrt(1.0 - b2 ** t)
            for p, g, m, v in zip(self.params, self.grads, self.m, self.v):
                ops.adam_step(p, g, m, v, lr_bc1, inv_sqrt_bc2, b1, b2, cfg.adam_eps)
        elif self.kind == OptimizerName.SGD:
            # clip_grad_norm_([A, B], max_norm=1.0) then SGD with momentum (gd.py:43-46)
            self.sumsq.zero_()
            if self.sum_group is not None:
                import torch.distributed as dist
                ops.grad_sumsq(self.grads[-1], self.sumsq)
                dist.all_reduce(self.sumsq, group=self.sum_group)
                for g in self.grads[:-1]:
                    ops.grad_sumsq(g, self.sumsq)
            else:
                for g in self.grads:
                    ops.grad_sumsq(g, self.sumsq)
            for p, g, buf in zip(self.params, self.grads, self.buf):
                ops.sgd_step(p, g, buf, cfg.learning_rate, cfg.momentum, t == 1, self.sumsq, 1.0)
        else:
            with torch.no_grad():
                for view, g in zip(self.views, self.grads):
                    view.grad = g[:, :view.shape[1]]
                self.torch_opt.step()


def _rows_csr(S_index, S_value, perm, m):
    """Support by global position in ``perm`` (local row of a block = position - k*bs):
    rowptr[m+1] over positions, entries {column, value bits}. Built once (GD keeps its
    partition for the whole run, gd.py:134-150)."""
    dev = S_value.device
    perm_inv = torch.empty_like(perm)
    perm_inv[perm] = torch.arange(m, device=dev)
    pos = perm_inv[S_index[0]]
    order = torch.sort(pos, stable=True).indices
    pos_sorted = pos[order]
    rowptr = torch.searchsorted(pos_sorted, torch.arange(m + 1, device=dev)).to(torch.int32)
    ent = torch.stack([S_index[1][order].to(torch.int32),
                       S_value[order].to(torch.float32).view(torch.int32)], dim=1).contiguous()
    return rowptr, ent


class GDState:
    """Device state of one GD run: padded factors and gradients, the optimizer, the fixed block
    partition with both CSR views of S, and the evaluation accumulators."""

    def __init__(self, S_index: Tensor, S_value: Tensor, m: int, n: int, cfg: SumacConfig,
                 A: Tensor, B: Tensor, gen_blocks, gen_loader):
        dev = cfg.device
        self.cfg = cfg
        self.d = d = cfg.rank
        self.Dp = Dp = ops.padded_rank(d)
        self.prec = cfg.precision()
        self.Ap = ops.pad_factor(A.detach().to(torch.float32), Dp)
        self.Bp = ops.pad_factor(B.detach().to(torch.float32), Dp)
        self.gA = torch.zeros_like(self.Ap)
        self.gB = torch.zeros_like(self.Bp)
        self.opt = _Optimizer(cfg, [self.Ap, self.Bp], [self.gA, self.gB], d)
        nb = cfg.num_blocks
        perm = draw_perm(m, gen_blocks, dev)     # one partition for the whole run (datasets.py:34)
        bs = (m + nb - 1) // nb
        self.dir_b = SparseDirection(S_index[0], S_index[1], S_value, m, n, nb)
        self.dir_b.rebuild(perm)                 # by column j, entries {local row, S}
        rowptr_pos, self.ent_pos = _rows_csr(S_index, S_value, perm, m)
        self.blocks = []
        for k in range(nb):
            rows = perm[k * bs:min(m, (k + 1) * bs)]
            self.blocks.append((rows, self.dir_b.block_rowptr(k),
                                rowptr_pos[k * bs:k * bs + rows.numel() + 1]))
        self.loader = DataLoader(list(range(nb)), batch_size=cfg.batch_blocks,
                                 shuffle=cfg.shuffle_blocks, collate_fn=lambda b: b,
                                 generator=gen_loader)
        self.sum_v = float(S_value.double().sum().item())
        self.s_norm = float(torch.linalg.norm(S_value.double()).item())
        self.terms = torch.zeros(8, dtype=torch.float64, device=dev)

    def epoch(self, report: bool) -> None:
        """One pass over the blocks in loader order (training/gd.py:160-204): per batch the loss
        terms (report epochs, before the step), the block gradients, one optimizer step."""
        d, prec = self.d, self.prec
        Ap, Bp, gA, gB = self.Ap, self.Bp, self.gA, self.gB
        if report:
            self.terms.zero_()
        for batch in self.loader:
            if report:
                for k in batch:
                    rows, rp_b, _ = self.blocks[k]
                    if rows.numel() > 0:
                        ops.block_loss_terms(Ap, Bp, d, rows, rp_b, self.dir_b.ent, self.terms, 1,
                                             prec)
            ops.fill_zero(gA)
            first = True
            for k in batch:
                rows, rp_b, rp_a = self.blocks[k]
                if rows.numel() == 0:
                    continue
                ops.gd_block_grad(Ap, Bp, d, rows, rp_b, self.dir_b.ent, rp_a, self.ent_pos, gA,
                                  gB, 0 if first else 1, prec)
                first = False
            if first:
                ops.fill_zero(gB)
            self.opt.step()

    def report_metrics(self) -> tuple[float, float, float]:
        return gd_epoch_metrics(self.terms, self.sum_v, self.s_norm)


def gd_epoch_metrics(terms: Tensor, sum_v: float, s_norm: float) -> tuple[float, float, float]:
    """(rmse, jacc, cost) of an epoch's accumulated block loss terms (eval.py:57-108)."""
    t = terms.cpu().tolist()
    sum_sr, sum_sr2, obs_sq, res_m, res_l, jnum = t[:6]
    total_errz = sum_sr2 - obs_sq + res_l
    total_mse = sum_sr2 - obs_sq + res_m
    jacc = 1.0 - jnum / (sum_v + sum_sr - jnum)
    rmse = math.sqrt(max(total_mse, 0.0)) / (s_norm + 1e-16)
    errZ = math.sqrt(max(total_errz, 0.0)) / (s_norm + 1e-16)
    return rmse, jacc, errZ


def GD_loop(S_index: Tensor, S_value: Tensor, m: int, n: int, cfg: SumacConfig,
            A_init: Tensor | None = None, B_init: Tensor | None = None):
    assert cfg.num_blocks is not None and cfg.device is not None
    dev = cfg.device
    gen, gen_blocks, gen_loader = cfg.get_generator()
    S_index = S_index.to(dev)
    S_value = S_value.to(dev)
    d = cfg.rank
    if A_init is None or B_init is None:
        A, B = init_salsa_factors(S_index, S_value, m, n, d, gen)
    else:
        A, B = A_init.to(dev).clone(), B_init.to(dev).clone()
    st = GDState(S_index, S_value, m, n, cfg, A, B, gen_blocks, gen_loader)
    evaluator = Evaluator(S_index, S_value, d, st.prec)
    rmse, jacc, errZ = evaluator(st.Ap, st.Bp)
    if cfg.verbose:
        print(f"[epoch 0/{cfg.max_iterations}]: cost = {errZ:.6f}, rmse = {rmse:.6f}, "
              f"jacc = {jacc:.6f}, time = 0.0000s")
    hist = {"cost": [], "rmse": [], "jacc": [], "time": []}
    t0 = time.time()
    for epoch in range(1, cfg.max_iterations + 1):
        report = epoch % cfg.eval_interval == 0
        st.epoch(report)
        if report:
            rmse, jacc, errZ = st.report_metrics()
            elapsed = time.time() - t0
            hist["cost"].append(errZ)
            hist["rmse"].append(rmse)
            hist["jacc"].append(jacc)
            hist["time"].append(elapsed)
            if cfg.verbose:
                print(f"[epoch {epoch}/{cfg.max_iterations}]: cost = {errZ:.6f}, "
                      f"rmse = {rmse:.6f}, jacc = {jacc:.6f}, time = {elapsed:.4f}s")
    _native.raise_device_error(dev)
    total = time.time() - t0
    if cfg.verbose:
        print(f"\nTotal elapsed time: {total:.2f} sec")
    rmse, jacc, errZ = evaluator(st.Ap, st.Bp)
    if cfg.verbose:
        print(f"EVAL: cost={errZ:.6f}, rmse={rmse:.6f}, jacc={jacc:.6f}, time={total:.4f}s")
    return st.Ap[:, :st.d].contiguous(), st.Bp[:, :st.d].contiguous(), hist
