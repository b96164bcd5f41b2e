"""Row-sharded SALSA over several GPUs (one process per GPU, torch.distributed with NCCL).

The reference's SALSA (src/sumac/training/salsa.py:212-355) updates, for every block k of an
iteration, all rows of B against the block's rows A_I of A, then all rows of A against the block's
rows B_J of B. Every row's update depends only on its own row, on the block rows of the fixed factor
and on that row's entries of S (salsa.py:84-166). So the work shards by rows with no partial sums:

* rank r owns the contiguous rows [lo, hi) of A and of B (and their momenta), and keeps, for each
  update direction, the entries of S whose updated row it owns (their fixed-row index stays global);
* before a block update, the block rows of the fixed factor (b x Dp, ~90 KB at C4's shapes) are
  assembled on every rank: each rank writes the rows it owns into a zero buffer and an allreduce
  (sum) completes it. With one nonzero contributor per element the sum is exact, so every rank
  holds bit-identical block rows, Gram matrix and least-squares map;
* each rank then runs the single-GPU block update (Gram + solve, fused product, finalize) on its
  own rows only.

Permutations come from the same seeded generators on every rank, so all ranks agree on the blocks
without communication. The factors are all-gathered only where the caller needs them whole
(evaluation, the end of the run).
"""
from __future__ import annotations

import time

import numpy as np
import torch
import torch.distributed as dist
from torch import Tensor

from . import _native, ops
from .config import OptimizerName, SumacConfig
from .data import SparseDirection
from .metrics import Evaluator
from .salsa import GRAPH_MIN_ITERATIONS_SHARDED, draw_perm, init_salsa_factors, unbias_values


def shard_range(total: int, rank: int, world: int) -> tuple[int, int]:
    """Rows [lo, hi) of a `total`-row factor owned by `rank` (balanced contiguous ranges)."""
    return total * rank // world, total * (rank + 1) // world


def split_direction(fixed: Tensor, out: Tensor, lo: int, hi: int) -> Tensor:
    """Mask of the entries whose updated row `out` lies in this rank's range [lo, hi)."""
    return (out >= lo) & (out < hi)


class SymmetricRows:
    """A [rows, Dp] staging buffer in symmetric memory (every rank can load every other rank's
    copy over NVLink), for the one-shot allreduce of assembled block rows: each rank reads its
    peers' buffers directly, a few microseconds for ~90 KB instead of an NCCL ring."""

    def __init__(self, rows: int, Dp: int, device, group=None):
        import torch.distributed._symmetric_memory as symm_mem
        self.group_name = (group or dist.group.WORLD).group_name
        self.buf = symm_mem.empty((rows, Dp), dtype=torch.float32, device=device)
        symm_mem.rendezvous(self.buf, self.group_name)

    def allreduce_into(self, b: int, out: Tensor) -> None:
        torch.ops.symm_mem.one_shot_all_reduce_out(self.buf[:b], "sum", self.group_name, out)


class P2PRows:
    """Block-row exchange over NVLink peer memory: a two-slot [2, rows, Dp] buffer and a flag
    array in symmetric memory on every rank, and a device exchange counter. Each exchange
    (`assemble`) is one native kernel: this rank stores the rows it owns into the current slot of
    every rank's buffer, then a flag barrier (one round, bounded wait) -- against the two barrier
    rounds and the reduction of a one-shot allreduce. Every rank makes the same sequence of calls;
    `pad_even` keeps the number of calls per iteration even, so that the slots a captured CUDA
    graph bakes in stay right on every replay."""

    def __init__(self, rows: int, Dp: int, device, group=None):
        import torch.distributed._symmetric_memory as symm_mem
        g = group or dist.group.WORLD
        name = g.group_name
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        self.rows, self.Dp = rows, Dp
        self.buf = symm_mem.empty((2, rows, Dp), dtype=torch.float32, device=device)
        hb = symm_mem.rendezvous(self.buf, name)
        self.flags = symm_mem.empty((self.world,), dtype=torch.int32, device=device)
        hf = symm_mem.rendezvous(self.flags, name)
        self.flags.zero_()
        self.buf.zero_()
        ob = self.buf.data_ptr() - hb.buffer_ptrs[self.rank]
        of = self.flags.data_ptr() - hf.buffer_ptrs[self.rank]
        self.peer_bufs = torch.tensor([p + ob for p in hb.buffer_ptrs], dtype=torch.int64,
                                      device=device)
        self.peer_flags = torch.tensor([p + of for p in hf.buffer_ptrs], dtype=torch.int64,
                                       device=device)
        self.epoch = torch.zeros(1, dtype=torch.int32, device=device)
        self.calls = 0
        self.empty_rows = torch.zeros(1, dtype=torch.int64, device=device)
        torch.cuda.synchronize(device)
        dist.barrier(group=group)  # every rank's flags are zero before anyone signals

    def assemble(self, local: Tensor, lo: int, hi: int, rows: Tensor) -> Tensor:
        """F[rows] (the assembled block rows) on every rank, as a view of the current slot."""
        b = rows.numel()
        self.calls += 1
        ops.assemble_rows_p2p(local, lo, hi, rows, b, self.rows * self.Dp, self.peer_bufs,
                              self.peer_flags, self.epoch, self.rank, self.world)
        return self.buf[self.calls & 1, :b]

    def pad_even(self, local: Tensor) -> None:
        if self.calls & 1:
            self.calls += 1
            ops.assemble_rows_p2p(local, 0, 0, self.empty_rows, 0, self.rows * self.Dp,
                                  self.peer_bufs, self.peer_flags, self.epoch, self.rank,
                                  self.world)


def make_p2p_rows(rows: int, Dp: int, device, group=None):
    """P2PRows on CUDA when symmetric memory is available, else None."""
    if device.type != "cuda":
        return None
    # ranks spinning on each other's flags must each have a GPU of their own
    ids = [None] * dist.get_world_size(group)
    dist.all_gather_object(ids, str(torch.cuda.get_device_properties(device).uuid), group=group)
    if len(set(ids)) != len(ids):
        return None
    try:
        return P2PRows(rows, Dp, device, group)
    except Exception:  # no peer access or no symmetric-memory backend
        return None


def make_symmetric_rows(rows: int, Dp: int, device, group=None):
    """SymmetricRows on CUDA when symmetric memory is available, else None (NCCL allreduce)."""
    if device.type != "cuda":
        return None
    try:
        return SymmetricRows(rows, Dp, device, group)
    except Exception:  # no peer access or no symmetric-memory backend: NCCL allreduce
        return None


def assemble_rows(local: Tensor, lo: int, hi: int, rows: Tensor, out: Tensor, group=None,
                  sym: SymmetricRows | None = None) -> None:
    """out[p] = F[rows[p]] for a factor F row-sharded over the group, this rank holding
    F[lo:hi] as `local`: the rows this rank owns are written, the others are zero, and an
    allreduce(sum) completes the buffer on every rank (exact: one nonzero term per element).
    With `sym`, the rows are staged in symmetric memory and reduced by a one-shot allreduce;
    otherwise by NCCL (or gloo on the CPU). No host synchronisation: graph-capturable."""
    b = rows.numel()
    if out.is_cuda:
        stage = sym.buf[:b] if sym is not None else out
        ops.gather_owned_rows(local, lo, hi, rows, stage)
        if sym is not None:
            sym.allreduce_into(b, out)
            return
    else:  # the CPU (gloo) path of the host-logic tests
        idx = (rows - lo).clamp(0, max(hi - lo - 1, 0))
        own = ((rows >= lo) & (rows < hi)).unsqueeze(1)
        torch.where(own, local[idx], torch.zeros((), dtype=local.dtype, device=local.device),
                    out=out)
    dist.all_reduce(out, group=group)


def gather_rows(local: Tensor, total: int, group=None) -> Tensor:
    """All-gather a row-sharded factor (contiguous balanced shards) into the whole factor."""
    world = dist.get_world_size(group)
    rmax = max(shard_range(total, r, world)[1] - shard_range(total, r, world)[0]
               for r in range(world))
    buf = torch.zeros((rmax,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    buf[:local.shape[0]] = local
    parts = [torch.empty_like(buf) for _ in range(world)]
    dist.all_gather(parts, buf, group=group)
    return torch.cat([parts[r][:shard_range(total, r, world)[1] - shard_range(total, r, world)[0]]
                      for r in range(world)])


class ShardedSalsaState:
    """Device state of one rank of a row-sharded SALSA run."""

    def __init__(self, S_index: Tensor, S_value: Tensor, m: int, n: int, cfg: SumacConfig,
                 A: Tensor, B: Tensor, group=None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.d = cfg.rank
        self.Dp = ops.padded_rank(self.d)
        self.m, self.n = m, n
        self.nb = cfg.num_blocks
        self.prec = cfg.precision()
        self.ra = shard_range(m, self.rank, self.world)
        self.rb = shard_range(n, self.rank, self.world)
        if self.ra[1] <= self.ra[0] or self.rb[1] <= self.rb[0]:
            raise ValueError(f"more ranks ({self.world}) than rows of a factor ({m} x {n})")
        dev = S_value.device
        self.Ap = ops.pad_factor(A[self.ra[0]:self.ra[1]].to(torch.float32), self.Dp)
        self.Bp = ops.pad_factor(B[self.rb[0]:self.rb[1]].to(torch.float32), self.Dp)
        self.dA = torch.zeros_like(self.Ap)
        self.dB = torch.zeros_like(self.Bp)
        i, j = S_index[0], S_index[1]
        # B-update: fixed = rows of A (global index), updated = this rank's rows of B
        kb = split_direction(i, j, *self.rb)
        self.dir_b = SparseDirection(i[kb], j[kb] - self.rb[0], S_value[kb], m,
                                     self.rb[1] - self.rb[0], self.nb)
        # A-update: fixed = rows of B (global index), updated = this rank's rows of A
        ka = split_direction(j, i, *self.ra)
        self.dir_a = SparseDirection(j[ka], i[ka] - self.ra[0], S_value[ka], n,
                                     self.ra[1] - self.ra[0], self.nb)
        self.FI_b = torch.zeros((self.dir_b.block_size, self.Dp), dtype=torch.float32, device=dev)
        self.FI_a = torch.zeros((self.dir_a.block_size, self.Dp), dtype=torch.float32, device=dev)
        self.ident = torch.arange(max(self.dir_a.block_size, self.dir_b.block_size),
                                  dtype=torch.int64, device=dev)
        self.p2p = make_p2p_rows(max(self.dir_a.block_size, self.dir_b.block_size), self.Dp,
                                 dev, group)
        self.sym = None if self.p2p is not None else make_symmetric_rows(
            max(self.dir_a.block_size, self.dir_b.block_size), self.Dp, dev, group)
        self.momentum = float(cfg.momentum)
        self.lrate = float(np.float32(cfg.learning_rate))
        self.unbias = torch.empty(self.nb, dtype=torch.float32, device=dev)
        self.unbias_host = torch.empty(self.nb, dtype=torch.float32).pin_memory()
        self.perm_r = torch.empty(m, dtype=torch.int64, device=dev)
        self.perm_c = torch.empty(n, dtype=torch.int64, device=dev)
        L = _native.lib()
        self.ws_b = ops._ws(dev, L.sumac_salsa_update_workspace_bytes(
            self.rb[1] - self.rb[0], self.dir_b.block_size, self.d, self.prec), "salsa_b")
        self.ws_a = ops._ws(dev, L.sumac_salsa_update_workspace_bytes(
            self.ra[1] - self.ra[0], self.dir_a.block_size, self.d, self.prec), "salsa_a")
        self.use_graph = True
        self.graph = None
        self.eager_done = False
        self.graph_launches = 0
        self.replayed_launches = 0

    def iteration(self, it: int, perm_r: Tensor, perm_c: Tensor) -> None:
        """One SALSA iteration on this rank's rows: eager the first time, then replays of a CUDA
        graph of the whole iteration (CSR rebuilds, assemblies with their allreduces, updates)."""
        nb = self.nb
        self.unbias_host.copy_(torch.from_numpy(unbias_values(self.momentum, 1 + (it - 1) * nb, nb)))
        self.unbias.copy_(self.unbias_host, non_blocking=True)
        if not self.use_graph or self.graph is None:
            if self.use_graph and self.eager_done:
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
            self._body(perm_r, perm_c)
            self.eager_done = True
            return
        self.perm_r.copy_(perm_r)
        self.perm_c.copy_(perm_c)
        self.graph.replay()
        self.replayed_launches += self.graph_launches

    def _body(self, perm_r: Tensor, perm_c: Tensor) -> None:
        self.dir_b.rebuild(perm_r)
        self.dir_a.rebuild(perm_c)
        for k in range(self.nb):
            rows = self.dir_b.block_rows(perm_r, k)
            b = rows.numel()
            if b > 0:
                FI = self._assemble(self.Ap, self.ra, rows, self.FI_b[:b])
                ops.salsa_block_update(FI, self.ident[:b], self.Bp, self.dB, self.d,
                                       self.dir_b.block_rowptr(k), self.dir_b.ent, self.momentum,
                                       self.lrate, self.unbias[k:k + 1], self.prec, self.ws_b)
            rows = self.dir_a.block_rows(perm_c, k)
            b = rows.numel()
            if b > 0:
                FI = self._assemble(self.Bp, self.rb, rows, self.FI_a[:b])
                ops.salsa_block_update(FI, self.ident[:b], self.Ap, self.dA, self.d,
                                       self.dir_a.block_rowptr(k), self.dir_a.ent, self.momentum,
                                       self.lrate, self.unbias[k:k + 1], self.prec, self.ws_a)
        if self.p2p is not None:
            self.p2p.pad_even(self.Ap)

    def _assemble(self, local: Tensor, rng, rows: Tensor, out: Tensor) -> Tensor:
        if self.p2p is not None:
            return self.p2p.assemble(local, rng[0], rng[1], rows)
        assemble_rows(local, rng[0], rng[1], rows, out, self.group, self.sym)
        return out

    def factors(self) -> tuple[Tensor, Tensor]:
        """The whole factors (all-gathered), on every rank."""
        A = gather_rows(self.Ap, self.m, self.group)[:, :self.d].contiguous()
        B = gather_rows(self.Bp, self.n, self.group)[:, :self.d].contiguous()
        return A, B


def sharded_salsa_loop(S_index: Tensor, S_value: Tensor, m: int, n: int, cfg: SumacConfig,
                       A_init: Tensor | None = None, B_init: Tensor | None = None, group=None):
    """salsa_loop with the rows sharded over the process group: same schedule, generators and
    history as the single-GPU loop; every rank returns the whole factors."""
    assert cfg.num_blocks is not None and cfg.device is not None
    gen, gen_rows, gen_cols = cfg.get_generator()
    dev = cfg.device
    S_index = S_index.to(dev)
    S_value = S_value.to(dev)
    if A_init is None or B_init is None:
        A, B = init_salsa_factors(S_index, S_value, m, n, cfg.rank, gen)
    else:
        A, B = A_init.to(dev), B_init.to(dev)
    st = ShardedSalsaState(S_index, S_value, m, n, cfg, A, B, group)
    st.use_graph = cfg.max_iterations >= GRAPH_MIN_ITERATIONS_SHARDED
    evaluator = Evaluator(S_index, S_value, cfg.rank, st.prec)
    draw_perm(m, gen_rows, dev)
    draw_perm(n, gen_cols, dev)
    rmse, jacc, errZ = evaluator(ops.pad_factor(A, st.Dp), ops.pad_factor(B, st.Dp))
    verbose = cfg.verbose and st.rank == 0
    if verbose:
        print(f"[epoch 0/{cfg.max_iterations}]: cost = {errZ:.6f}, rmse = {rmse:.6f}, "
              f"jacc = {jacc:.6f}, time = 0.0000s")
    hist = {"cost": [], "rmse": [], "jacc": [], "time": []}
    t0 = time.time()
    for it in range(1, cfg.max_iterations + 1):
        perm_r = draw_perm(m, gen_rows, dev)
        perm_c = draw_perm(n, gen_cols, dev)
        st.iteration(it, perm_r, perm_c)
        if cfg.eval_interval is not None and it % cfg.eval_interval == 0:
            A, B = st.factors()
            rmse, jacc, errZ = evaluator(ops.pad_factor(A, st.Dp), ops.pad_factor(B, st.Dp))
            _native.raise_device_error(dev)
            elapsed = time.time() - t0
            hist["cost"].append(errZ)
            hist["rmse"].append(rmse)
            hist["jacc"].append(jacc)
            hist["time"].append(elapsed)
            if verbose:
                print(f"[epoch {it}/{cfg.max_iterations}]: cost = {errZ:.6f}, rmse = {rmse:.6f}, "
                      f"jacc = {jacc:.6f}, time = {elapsed:.4f}s")
    _native.raise_device_error(dev)
    A, B = st.factors()
    return A, B, hist


# ---------------------------------------------------------------------------------------------
# GD (training/gd.py:110-253): every step's row block is split over the ranks
# ---------------------------------------------------------------------------------------------
def subblock_bounds(m: int, nb: int, k: int, rank: int, world: int) -> tuple[int, int]:
    """Positions [lo, hi) (within block k of the fixed partition) of this rank's sub-block."""
    bs = (m + nb - 1) // nb
    bk = max(0, min(bs, m - k * bs))
    return bk * rank // world, bk * (rank + 1) // world


def virtual_positions(pos: Tensor, m: int, nb: int, rank: int, world: int) -> Tensor:
    """For global positions `pos` in the partition permutation: the rank-local virtual position
    k * bsub + (t - lo_k) when the position falls in this rank's sub-block of its block k
    (t = pos - k * bs), else -1. Sub-blocks occupy whole virtual blocks of bsub = ceil(bs / world)
    slots, so the single-GPU per-block CSR builder (block = vpos / bsub) works unchanged."""
    bs = (m + nb - 1) // nb
    bsub = (bs + world - 1) // world
    k = torch.div(pos, bs, rounding_mode="floor")
    t = pos - k * bs
    bk = torch.clamp(m - k * bs, max=bs)
    lo = torch.div(bk * rank, world, rounding_mode="floor")
    hi = torch.div(bk * (rank + 1), world, rounding_mode="floor")
    own = (t >= lo) & (t < hi)
    return torch.where(own, k * bsub + (t - lo), torch.full_like(pos, -1))


def combine_block_grads(gA: Tensor, gB: Tensor, block_rows: list[Tensor], gbuf: Tensor,
                        group=None, reduce_b: bool = True) -> None:
    """Complete the gradients of one GD step whose row blocks were split over the ranks: each
    rank holds grad A on the rows of its sub-blocks (zero on the other rows of the blocks) and a
    partial grad B over its sub-blocks' entries. grad B is the sum of the partials (allreduce);
    the blocks' rows of grad A are disjoint between ranks, so their sum (an allreduce of the
    gathered rows) is exact. Afterwards every rank holds the whole step's gradients (grad B
    only with reduce_b; otherwise the caller reduce-scatters it)."""
    if reduce_b:
        dist.all_reduce(gB, group=group)
    for full in block_rows:
        b = full.numel()
        if b == 0:
            continue
        torch.index_select(gA, 0, full, out=gbuf[:b])
        dist.all_reduce(gbuf[:b], group=group)
        gA.index_copy_(0, full, gbuf[:b])


class ShardedGDState:
    """One rank of a GD run whose row blocks are split over the ranks. The factors, their
    gradients and the optimizer state are replicated; each rank computes the gradients of its
    sub-block (its rows of grad A, a partial grad B), grad B is allreduced (sum) and the block's
    rows of grad A are completed by an exact allreduce, then every rank takes the same optimizer
    step. Same partition, loader order and optimizer as GDState."""

    def __init__(self, S_index: Tensor, S_value: Tensor, m: int, n: int, cfg: SumacConfig,
                 A: Tensor, B: Tensor, gen_blocks, gen_loader, group=None):
        from torch.utils.data import DataLoader
        from .gd import _Optimizer
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        dev = cfg.device
        self.cfg = cfg
        self.d = d = cfg.rank
        self.Dp = Dp = ops.padded_rank(d)
        self.prec = cfg.precision()
        self.Ap = ops.pad_factor(A.detach().to(torch.float32), Dp)
        self.gA = torch.zeros_like(self.Ap)
        # B, grad B: n rows padded to a multiple of the world size, so that grad B can be
        # reduce-scattered into equal row slices and B all-gathered back from them
        chunk = (n + self.world - 1) // self.world
        self.Bfull = torch.zeros((chunk * self.world, Dp), dtype=torch.float32, device=dev)
        self.Bfull[:n, :d] = B.detach().to(torch.float32)
        self.gBfull = torch.zeros_like(self.Bfull)
        self.Bp, self.gB = self.Bfull[:n], self.gBfull[:n]
        # ZeRO-1 for B (Adam, AdamW, SGD: elementwise steps): each rank steps only its slice of B
        # and keeps only that slice's optimizer state; Muon (whole-matrix step) stays replicated
        self.zero_b = cfg.optimizer in (OptimizerName.ADAM, OptimizerName.ADAMW, OptimizerName.SGD)
        if self.zero_b:
            self.Bslice = self.Bfull[self.rank * chunk:(self.rank + 1) * chunk]
            self.gBslice = torch.zeros_like(self.Bslice)
            self.opt = _Optimizer(cfg, [self.Ap, self.Bslice], [self.gA, self.gBslice], d,
                                  sum_group=group)
        else:
            self.opt = _Optimizer(cfg, [self.Ap, self.Bp], [self.gA, self.gB], d)
        self.m, self.n = m, n
        nb = self.nb = cfg.num_blocks
        perm = draw_perm(m, gen_blocks, dev)     # the same partition on every rank
        bs = (m + nb - 1) // nb
        bsub = (bs + self.world - 1) // self.world
        nv = nb * bsub
        perm_inv = torch.empty_like(perm)
        perm_inv[perm] = torch.arange(m, device=dev)
        vpos = virtual_positions(perm_inv[S_index[0]], m, nb, self.rank, self.world)
        keep = vpos >= 0
        vp, cols, vals = vpos[keep], S_index[1][keep], S_value[keep]
        # by column j (entries {row within the sub-block, S}): the CSR builder on the identity
        # permutation of the virtual positions
        self.dir_b = SparseDirection(vp, cols, vals, nv, n, nb)
        self.dir_b.rebuild(torch.arange(nv, dtype=torch.int64, device=dev))
        # by row within the sub-block (entries {j, S}), in the support's original order
        order = torch.sort(vp, stable=True).indices
        self.rowptr_v = torch.searchsorted(vp[order], torch.arange(nv + 1, device=dev)).to(torch.int32)
        self.ent_v = torch.stack([cols[order].to(torch.int32),
                                  vals[order].to(torch.float32).view(torch.int32)], 1).contiguous()
        self.blocks = []
        for k in range(nb):
            lo, hi = subblock_bounds(m, nb, k, self.rank, self.world)
            full = perm[k * bs:min(m, (k + 1) * bs)]
            self.blocks.append((full[lo:hi], full, self.dir_b.block_rowptr(k),
                                self.rowptr_v[k * bsub:k * bsub + (hi - lo) + 1]))
        self.gbuf = torch.zeros((bs, Dp), dtype=torch.float32, device=dev)
        self.loader = DataLoader(list(range(nb)), batch_size=cfg.batch_blocks,
                                 shuffle=cfg.shuffle_blocks, collate_fn=lambda b: b,
                                 generator=gen_loader)
        self.sum_v = float(S_value.double().sum().item())
        self.s_norm = float(torch.linalg.norm(S_value.double()).item())
        self.terms = torch.zeros(8, dtype=torch.float64, device=dev)

    def epoch(self, report: bool) -> None:
        d, prec = self.d, self.prec
        Ap, Bp, gA, gB = self.Ap, self.Bp, self.gA, self.gB
        if report:
            self.terms.zero_()
        for batch in self.loader:
            if report:
                for k in batch:
                    sub, _, rp_b, _ = self.blocks[k]
                    if sub.numel() > 0:
                        ops.block_loss_terms(Ap, Bp, d, sub, rp_b, self.dir_b.ent, self.terms, 1,
                                             prec)
            ops.fill_zero(gA)
            first = True
            for k in batch:
                sub, _, rp_b, rp_a = self.blocks[k]
                if sub.numel() == 0:
                    continue
                ops.gd_block_grad(Ap, Bp, d, sub, rp_b, self.dir_b.ent, rp_a, self.ent_v, gA, gB,
                                  0 if first else 1, prec)
                first = False
            if first:
                ops.fill_zero(gB)
            combine_block_grads(gA, gB, [self.blocks[k][1] for k in batch], self.gbuf,
                                self.group, reduce_b=not self.zero_b)
            if self.zero_b:
                # reduce-scatter grad B (sum) -> step this rank's slice -> all-gather B
                dist.reduce_scatter_tensor(self.gBslice, self.gBfull, group=self.group)
                self.opt.step()
                dist.all_gather_into_tensor(self.Bfull, self.Bslice, group=self.group)
            else:
                self.opt.step()
        if report:
            dist.all_reduce(self.terms, group=self.group)

    def report_metrics(self) -> tuple[float, float, float]:
        from .gd import gd_epoch_metrics
        return gd_epoch_metrics(self.terms, self.sum_v, self.s_norm)


def sharded_gd_loop(S_index: Tensor, S_value: Tensor, m: int, n: int, cfg: SumacConfig,
                    A_init: Tensor | None = None, B_init: Tensor | None = None, group=None):
    """GD_loop with every step's row block split over the process group; same schedule,
    generators and history; every rank returns the whole factors."""
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
    st = ShardedGDState(S_index, S_value, m, n, cfg, A, B, gen_blocks, gen_loader, group)
    evaluator = Evaluator(S_index, S_value, d, st.prec)
    rmse, jacc, errZ = evaluator(st.Ap, st.Bp)
    verbose = cfg.verbose and st.rank == 0
    if verbose:
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
            if verbose:
                print(f"[epoch {epoch}/{cfg.max_iterations}]: cost = {errZ:.6f}, "
                      f"rmse = {rmse:.6f}, jacc = {jacc:.6f}, time = {elapsed:.4f}s")
    _native.raise_device_error(dev)
    return st.Ap[:, :d].contiguous(), st.Bp[:, :d].contiguous(), hist
