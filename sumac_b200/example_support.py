"""Input loaders and result files of the reference's example scripts
(src/sumac/example_support/_example_shared.py:14-103): the same file formats, index conventions
and output files, so that a run of `examples/sumac_*.py` can be pointed at this library.

* `.mat` files: the sparse matrix stored under `S` (digits) or under the example's name
  (`bigrams`, `connectome`); bigram counts are divided by their row sums (+ the smallest normal
  float32, so that empty rows stay zero).
* other files: whitespace-separated text triplets `row col value` with 1-based indices; the shape is
  taken from the largest indices (square for `connectome`).
* `load_factorize_save` writes `AB.pt` ([A, B] via torch.save), `cost.pkl` (the history) and
  `opts.pkl` (the config's fields) under `save_path`.
"""
from __future__ import annotations

import os
import pickle
from typing import Literal

import numpy as np
import torch

from .config import SumacConfig

ExampleType = Literal["digits", "bigrams", "connectome"]


def make_paths(cfg: SumacConfig, etype: ExampleType) -> tuple[str, str | None]:
    """The output directory of a run (created) and the log file name (its directory created)."""
    parts = [f"sumac_rank={cfg.rank}", f"mom={cfg.momentum}", f"seed={cfg.seed}",
             f"iters={cfg.max_iterations}", f"nblocks={cfg.num_blocks}",
             f"learning_rate={cfg.learning_rate}", f"optim={cfg.optimizer.value}"]
    save_path = os.path.join(".", f"{etype}_{cfg.method.value}", "_".join(parts))
    os.makedirs(save_path, exist_ok=True)
    if cfg.log_filename is not None and os.path.dirname(cfg.log_filename):
        os.makedirs(os.path.dirname(cfg.log_filename), exist_ok=True)
    return save_path, cfg.log_filename


def _from_mat(filename: str, etype: ExampleType, dtype: torch.dtype):
    import scipy.io
    S = scipy.io.loadmat(filename)["S" if etype == "digits" else etype].tocoo()
    vals = S.data
    if etype == "bigrams":
        sums = np.asarray(S.sum(axis=1), dtype=np.float32).reshape(-1)
        vals = S.data.astype(np.float32) / (sums[S.row] + np.finfo(np.float32).tiny)
    index = torch.from_numpy(np.stack([S.row, S.col]).astype(np.int64))
    return int(S.shape[0]), int(S.shape[1]), index, torch.tensor(vals, dtype=dtype)


def _from_text(filename: str, etype: ExampleType):
    cols = np.loadtxt(filename, ndmin=2).T
    index = torch.tensor(cols[0:2], dtype=torch.long)
    values = torch.tensor(cols[2], dtype=torch.float)
    m = int(index[0].max().item())
    n = m if etype == "connectome" else int(index[1].max().item())
    return m, n, index - 1, values


def load_data(filename: str, etype: ExampleType, dtype: torch.dtype = torch.float32):
    """(m, n, S_index [2, nnz] int64 0-based, S_value [nnz])."""
    if filename.endswith(".mat"):
        return _from_mat(filename, etype, dtype)
    return _from_text(filename, etype)


def load_factorize_save(config: SumacConfig, etype: ExampleType, save_path: str):
    """Load `config.input_filename`, factorize it and write AB.pt, cost.pkl and opts.pkl."""
    from .sumac import sumac_factorize
    if config.input_filename is None:
        raise ValueError("config.input_filename is required")
    m, n, S_index, S_value = load_data(config.input_filename, etype, config.dtype)
    A, B, costs = sumac_factorize(S_index=S_index, S_value=S_value, shape=(m, n), config=config)
    torch.save([A, B], os.path.join(save_path, "AB.pt"))
    with open(os.path.join(save_path, "cost.pkl"), "wb") as f:
        pickle.dump(costs, f)
    with open(os.path.join(save_path, "opts.pkl"), "wb") as f:
        pickle.dump(vars(config), f)
    return A, B, costs
