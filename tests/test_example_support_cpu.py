"""The example scripts' loaders (src/sumac/example_support/_example_shared.py:44-87): text triplets
with 1-based indices, .mat matrices (bigram row normalisation), and the run directory name."""
import os

import numpy as np
import scipy.io
import scipy.sparse
import torch

from sumac_b200 import SumacConfig, SumacMethod
from sumac_b200.example_support import load_data, make_paths


def test_text_triplets_are_one_based(tmp_path):
    f = tmp_path / "s.txt"
    f.write_text("1 2 0.5\n3 1 2.0\n2 4 1.5\n")
    m, n, idx, val = load_data(str(f), "digits")
    assert (m, n) == (3, 4)
    assert idx.tolist() == [[0, 2, 1], [1, 0, 3]]
    assert val.dtype == torch.float32
    np.testing.assert_allclose(val.numpy(), [0.5, 2.0, 1.5])
    m, n, _, _ = load_data(str(f), "connectome")
    assert (m, n) == (3, 3)


def test_mat_digits_and_bigram_normalisation(tmp_path):
    S = scipy.sparse.coo_matrix((np.array([1.0, 3.0, 2.0]), (np.array([0, 0, 2]), np.array([1, 3, 0]))),
                                shape=(4, 5))
    scipy.io.savemat(tmp_path / "d.mat", {"S": S.tocsc()})
    scipy.io.savemat(tmp_path / "b.mat", {"bigrams": S.tocsc()})
    m, n, idx, val = load_data(str(tmp_path / "d.mat"), "digits")
    assert (m, n) == (4, 5)
    got = {(int(i), int(j)): float(v) for i, j, v in zip(idx[0], idx[1], val)}
    assert got == {(0, 1): 1.0, (0, 3): 3.0, (2, 0): 2.0}
    _, _, idx, val = load_data(str(tmp_path / "b.mat"), "bigrams")
    got = {(int(i), int(j)): float(v) for i, j, v in zip(idx[0], idx[1], val)}
    np.testing.assert_allclose([got[(0, 1)], got[(0, 3)], got[(2, 0)]], [0.25, 0.75, 1.0],
                               rtol=1e-6)


def test_make_paths(tmp_path, monkeypatch):
    monkeypatch.chdir(tmp_path)
    cfg = SumacConfig(method=SumacMethod.SALSA, rank=7, seed=3, max_iterations=5, num_blocks=4,
                      verbose=False, log_filename="logs/run.log")
    path, log = make_paths(cfg, "digits")
    assert os.path.isdir(path) and os.path.isdir("logs")
    assert path == os.path.join(".", "digits_" + cfg.method.value,
                                f"sumac_rank=7_mom={cfg.momentum}_seed=3_iters=5_nblocks=4_"
                                f"learning_rate={cfg.learning_rate}_optim={cfg.optimizer.value}")
    assert log == "logs/run.log"
