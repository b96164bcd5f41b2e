"""Generate the golden fixtures in this folder by running the reference (flatironinstitute/sumac)
on the CPU.

Run from the repository root, in a container that has the reference checked out:

    SUMAC_REFERENCE_SRC=<path to sumac>/src python tests/golden/make_golden.py

It imports the reference read-only, with TorchDynamo disabled (its torch.compile wrappers then run
eagerly on the CPU) and ``AutotuneMode.DISABLE`` (CPU tensors always take the reference's torch
fallbacks, ``kernels/tuning/autotune.py:181-191``). Every fixture is a small ``.npz`` holding the
inputs and the reference's outputs. The GPU box never runs this script; the tests only read the
``.npz`` files.
"""
from __future__ import annotations

import os
import sys

os.environ.setdefault("TORCHDYNAMO_DISABLE", "1")
if "SUMAC_REFERENCE_SRC" not in os.environ:
    sys.exit("set SUMAC_REFERENCE_SRC to the reference's src directory (see the docstring)")
sys.path.insert(0, os.environ["SUMAC_REFERENCE_SRC"])

import numpy as np  # noqa: E402
import torch  # noqa: E402

from sumac import AutotuneMode, SumacConfig, SumacMethod, sumac_factorize  # noqa: E402
from sumac.datasets import StochasticRowBlockDataset  # noqa: E402
from sumac.eval import block_loss_and_pred, eval as ref_eval  # noqa: E402
from sumac.kernels.tuning import AutotuneReluBatReduce, kernel_autotune_options  # noqa: E402
from sumac.kernels.tuning.relu_bat_c.relu_bat_c_base import relu_bat_c_fallback  # noqa: E402
from sumac.kernels.tuning.relu_bat_reduce.relu_bat_reduce import relu_bat_reduce_fallback  # noqa: E402
from sumac.training import salsa  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))


def save(name, **arrays):
    conv = {}
    for k, v in arrays.items():
        if isinstance(v, torch.Tensor):
            v = v.detach().cpu().numpy()
        conv[k] = np.asarray(v)
    np.savez_compressed(os.path.join(OUT, name + ".npz"), **conv)


def random_sparse(gen, m, n, density, empty_rows=(), empty_cols=()):
    mask = torch.rand(m, n, generator=gen) < density
    for r in empty_rows:
        mask[r] = False
    for c in empty_cols:
        mask[:, c] = False
    idx = mask.nonzero().T.contiguous()
    vals = 0.05 + torch.rand(idx.shape[1], generator=gen)
    return idx, vals.float()


class RefReluBatC:
    """Stand-in for the tuned relu_bat_c kernel: the reference's own fallback formula."""

    def __call__(self, tup):
        A, B, C = tup
        return relu_bat_c_fallback(A, B, C)

    def resolve_decision(self, *_):
        return None


def kernels():
    g = torch.Generator().manual_seed(11)
    for tag, (N, M, D) in {"a": (37, 150, 13), "b": (64, 200, 16), "c": (50, 130, 32)}.items():
        A = torch.randn(N, D, generator=g)
        B = torch.randn(M, D, generator=g)
        C = torch.randn(N, D, generator=g)
        Y = relu_bat_c_fallback(A, B, C)
        s1, s2 = relu_bat_reduce_fallback(B, A)
        save(f"relu_bat_c_{tag}", A=A, B=B, C=C, Y=Y, sum_sr=s1, sum_sr2=s2)


def lsq_steps():
    g = torch.Generator().manual_seed(12)
    b, M, d = 6, 9, 3
    A = torch.randn(b, d, generator=g, dtype=torch.float64)
    B = torch.randn(M, d, generator=g, dtype=torch.float64)
    dB = 0.1 * torch.randn(M, d, generator=g, dtype=torch.float64)
    P = torch.linalg.solve(A.T @ A, A.T).T
    pairs = torch.randperm(b * M, generator=g)[:17]
    edge_i, edge_j = pairs // M, pairs % M
    vals = 0.2 + torch.rand(17, generator=g, dtype=torch.float64)
    mu = torch.tensor(0.7, dtype=torch.float64)
    unbias = 1.0 - mu ** 5
    lr = torch.tensor(0.1, dtype=torch.float64)
    Bn, dBn = salsa.lsq_update_single_gpu(RefReluBatC(), Ar_dev=A, B_blk_dev=B, pinvAt_dev=P,
                                          dB_blk_dev=dB, edge_i=edge_i, edge_j=edge_j,
                                          blk_vals=vals, momentum=mu, unbias=unbias, lrate=lr)
    save("lsq_update", A=A, B=B, dB=dB, P=P, edge_i=edge_i, edge_j=edge_j, vals=vals,
         momentum=mu, unbias=unbias, lr=lr, B_new=Bn, dB_new=dBn)

    # batch update with shuffled fixed rows (salsa.py:119-166)
    m_fixed, n_upd, d = 11, 8, 3
    F = torch.randn(m_fixed, d, generator=g, dtype=torch.float64)
    B = torch.randn(n_upd, d, generator=g, dtype=torch.float64)
    dB = 0.1 * torch.randn(n_upd, d, generator=g, dtype=torch.float64)
    idx, vals = random_sparse(g, m_fixed, n_upd, 0.4)
    vals = vals.double()
    rows = torch.tensor([7, 2, 9, 0, 4], dtype=torch.long)
    in_blk = torch.isin(idx[0], rows)
    edge_idx = in_blk.nonzero().flatten()
    fn = getattr(salsa.batch_update_single_gpu, "_torchdynamo_orig_callable",
                 salsa.batch_update_single_gpu)
    Bn, dBn = fn(RefReluBatC(), S_idx_full=idx, S_val_full=vals, edge_idx=edge_idx, Factor_fixed=F,
                 row_indices=rows, B=B, dB=dB, momentum=mu, unbias=unbias, lrate=lr,
                 m_fixed=m_fixed)
    save("batch_update", F=F, B=B, dB=dB, S_index=idx, S_value=vals, rows=rows, edge_idx=edge_idx,
         momentum=mu, unbias=unbias, lr=lr, B_new=Bn, dB_new=dBn)


def partition():
    g = torch.Generator().manual_seed(13)
    m, n, nb = 57, 40, 5
    idx, vals = random_sparse(g, m, n, 0.2)
    gen = torch.Generator().manual_seed(101)
    ds = StochasticRowBlockDataset(idx, vals, m, nb, gen)
    perm = torch.cat(ds.block_row_indices)
    sets = [torch.sort(e)[0] for e in ds.block_edge_idx]
    counts = torch.tensor([len(s) for s in sets])
    save("partition", S_index=idx, S_value=vals, m=m, num_blocks=nb, perm=perm,
         edges=torch.cat(sets), counts=counts)


def metrics_and_gd_grad():
    g = torch.Generator().manual_seed(14)
    m, n, d, nb = 45, 38, 4, 3
    idx, vals = random_sparse(g, m, n, 0.25)
    A = torch.randn(m, d, generator=g)
    B = torch.randn(n, d, generator=g)
    gen = torch.Generator().manual_seed(5)
    ds = StochasticRowBlockDataset(idx, vals, m, nb, gen)
    loader = torch.utils.data.DataLoader(ds, batch_size=1, shuffle=False, collate_fn=lambda b: b)
    with kernel_autotune_options(mode=AutotuneMode.DISABLE, cache_dir="/tmp/sumac_golden",
                                 verbose=False):
        kern = AutotuneReluBatReduce()
        rmse, jacc, cost = ref_eval(kern, A, B, idx, vals, loader, device=torch.device("cpu"))
        rows0 = ds.block_row_indices[0]
        edge0 = ds.block_edge_idx[0]
        Ap = A.clone().requires_grad_(True)
        Bp = B.clone().requires_grad_(True)
        mse_b, sumsr_b, jacc_b, errz_b = block_loss_and_pred(kern, Ap, Bp, idx, vals, edge0, rows0)
        errz_b.backward()
    save("metrics", S_index=idx, S_value=vals, A=A, B=B, perm=torch.cat(ds.block_row_indices),
         num_blocks=nb, rmse=rmse, jacc=jacc, cost=cost)
    save("gd_block", S_index=idx, S_value=vals, A=A, B=B, rows=rows0, edge_idx=edge0,
         mse=mse_b, sum_sr=sumsr_b, jacc_num=jacc_b, errZ=errz_b, grad_A=Ap.grad, grad_B=Bp.grad)


def end_to_end():
    # SALSA, 3 iterations, warm start, two empty rows and one empty column (pruning path).
    g = torch.Generator().manual_seed(15)
    m, n, d, nb = 120, 90, 6, 4
    idx, vals = random_sparse(g, m, n, 0.15, empty_rows=(3, 77), empty_cols=(10,))
    A0 = torch.rand(m, d, generator=g)
    B0 = -torch.rand(n, d, generator=g)
    cfg = SumacConfig(method=SumacMethod.SALSA, rank=d, max_iterations=3, num_blocks=nb,
                      eval_interval=1, seed=0, verbose=False, learning_rate=0.5,
                      autotune=AutotuneMode.DISABLE, device=torch.device("cpu"))
    A, B, hist = sumac_factorize(S_index=idx, S_value=vals, shape=(m, n), A_init=A0, B_init=B0,
                                 config=cfg)
    save("e2e_salsa", S_index=idx, S_value=vals, m=m, n=n, rank=d, num_blocks=nb, iters=3,
         seed=0, lr=0.5, A0=A0, B0=B0, A=A, B=B, cost=hist["cost"], rmse=hist["rmse"],
         jacc=hist["jacc"])

    # GD with Adam, two blocks per batch, shuffled blocks.
    g = torch.Generator().manual_seed(16)
    m, n, d, nb = 100, 80, 5, 3
    idx, vals = random_sparse(g, m, n, 0.2)
    A0 = 0.5 * torch.rand(m, d, generator=g)
    B0 = 0.5 * torch.randn(n, d, generator=g)
    cfg = SumacConfig(method=SumacMethod.GD, rank=d, max_iterations=4, num_blocks=nb,
                      batch_blocks=2, shuffle_blocks=True, eval_interval=2, seed=3,
                      learning_rate=0.01, verbose=False, autotune=AutotuneMode.DISABLE,
                      device=torch.device("cpu"))
    A, B, hist = sumac_factorize(S_index=idx, S_value=vals, shape=(m, n), A_init=A0, B_init=B0,
                                 config=cfg)
    save("e2e_gd", S_index=idx, S_value=vals, m=m, n=n, rank=d, num_blocks=nb, iters=4, seed=3,
         lr=0.01, batch_blocks=2, A0=A0, B0=B0, A=A, B=B, cost=hist["cost"], rmse=hist["rmse"],
         jacc=hist["jacc"])


def c1_planted():
    """the planted 2000 x 1500 problem (bench.make_c1, deterministic numpy),
    GD with rank 8 for 50 iterations from the reference's own initialisation (no A_init/B_init),
    seed 0, on the CPU. The data are regenerated by the tests from bench.make_c1; the fixture keeps
    their size and checksum, the reference's initial factors (init_salsa_factors with the seed-0
    generator, as GD_loop draws them) and the run's history and final factors."""
    sys.path.insert(0, os.path.dirname(os.path.dirname(OUT)))
    from bench import make_c1
    from sumac.training.salsa import init_salsa_factors
    idx_np, val_np, (m, n) = make_c1()
    idx = torch.from_numpy(idx_np)
    vals = torch.from_numpy(val_np)
    assert torch.unique(idx[0]).numel() == m and torch.unique(idx[1]).numel() == n  # nothing pruned
    d, iters = 8, 50
    gen = torch.Generator(device="cpu").manual_seed(0)
    A0, B0 = init_salsa_factors(idx, vals, m, n, d, gen)
    cfg = SumacConfig(method=SumacMethod.GD, rank=d, max_iterations=iters, eval_interval=10,
                      seed=0, verbose=False, autotune=AutotuneMode.DISABLE,
                      device=torch.device("cpu"))
    A, B, hist = sumac_factorize(S_index=idx, S_value=vals, shape=(m, n), config=cfg)
    save("c1_gd", m=m, n=n, rank=d, iters=iters, seed=0, nnz=vals.numel(),
         value_sum=vals.double().sum(), A0=A0, B0=B0, A=A, B=B, cost=hist["cost"],
         rmse=hist["rmse"], jacc=hist["jacc"])


if __name__ == "__main__":
    torch.set_num_threads(4)
    kernels()
    lsq_steps()
    partition()
    metrics_and_gd_grad()
    end_to_end()
    c1_planted()
    print("golden fixtures written to", OUT, "with torch", torch.__version__)
