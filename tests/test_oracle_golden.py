"""Pins the CPU oracle (oracle/sumac_oracle.py) to golden vectors produced by the reference
(tests/golden/make_golden.py). CPU only."""
import numpy as np
import torch

from oracle import sumac_oracle as orc


def test_relu_bat_c_and_reduce(golden):
    for tag in "abc":
        g = golden(f"relu_bat_c_{tag}")
        Y = orc.relu_bat_c(g["A"], g["B"], g["C"])
        np.testing.assert_allclose(Y, g["Y"], rtol=1e-4, atol=1e-4)
        s1, s2 = orc.relu_bat_reduce(g["B"], g["A"])
        np.testing.assert_allclose([s1, s2], [g["sum_sr"], g["sum_sr2"]], rtol=1e-5)


def test_lsq_update(golden):
    g = golden("lsq_update")
    Bn, dBn = orc.lsq_update(g["A"], g["B"], g["P"], g["dB"], g["edge_i"], g["edge_j"], g["vals"],
                             float(g["momentum"]), float(g["unbias"]), float(g["lr"]))
    np.testing.assert_allclose(Bn, g["B_new"], rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(dBn, g["dB_new"], rtol=1e-12, atol=1e-12)


def test_block_update(golden):
    g = golden("batch_update")
    Bn, dBn = orc.block_update(g["F"], g["rows"], g["B"], g["dB"], g["S_index"], g["S_value"],
                               g["edge_idx"], float(g["momentum"]), float(g["unbias"]), float(g["lr"]))
    np.testing.assert_allclose(Bn, g["B_new"], rtol=1e-10, atol=1e-12)
    np.testing.assert_allclose(dBn, g["dB_new"], rtol=1e-10, atol=1e-12)


def test_partition_sets(golden):
    g = golden("partition")
    sets = orc.block_edge_sets(g["perm"], g["S_index"][0], int(g["num_blocks"]))
    counts = np.array([len(s) for s in sets])
    np.testing.assert_array_equal(counts, g["counts"])
    np.testing.assert_array_equal(np.concatenate(sets), g["edges"])


def test_block_csr_matches_partition(golden):
    g = golden("partition")
    idx, vals, nb = g["S_index"], g["S_value"], int(g["num_blocks"])
    M = int(idx[1].max()) + 1
    rowptr, local, v = orc.block_csr(g["perm"], idx[0], idx[1], vals, nb, M)
    sets = orc.block_edge_sets(g["perm"], idx[0], nb)
    bs, blk, loc, rows = orc.block_partition(g["perm"], idx[0], nb)
    for k in range(nb):
        lo, hi = rowptr[k * M], rowptr[(k + 1) * M]
        assert hi - lo == len(sets[k])
        got = set()
        for j in range(M):
            for e in range(rowptr[k * M + j], rowptr[k * M + j + 1]):
                got.add((int(rows[k][local[e]]), j, float(v[e])))
        want = {(int(idx[0, e]), int(idx[1, e]), float(vals[e])) for e in sets[k]}
        assert got == want


def test_metrics(golden):
    g = golden("metrics")
    nb = int(g["num_blocks"])
    _, _, _, rows = orc.block_partition(g["perm"], g["S_index"][0], nb)
    rmse, jacc, cost = orc.evaluate(g["A"], g["B"], g["S_index"], g["S_value"], rows)
    np.testing.assert_allclose([rmse, jacc, cost], [g["rmse"], g["jacc"], g["cost"]], rtol=1e-5)
    t = orc.eval_terms(g["A"], g["B"], g["S_index"], g["S_value"])
    np.testing.assert_allclose(orc.metrics_from_terms(t), [g["rmse"], g["jacc"], g["cost"]], rtol=1e-5)


def test_gd_block_grad(golden):
    g = golden("gd_block")
    idx, rows, eidx = g["S_index"], g["rows"], g["edge_idx"]
    local = np.full(g["A"].shape[0], -1)
    local[rows] = np.arange(rows.size)
    errZ, gA_I, gB = orc.gd_block_grad(g["A"][rows], g["B"], local[idx[0, eidx]], idx[1, eidx],
                                       g["S_value"][eidx])
    np.testing.assert_allclose(errZ, g["errZ"], rtol=1e-5)
    gA = np.zeros_like(g["A"], dtype=np.float64)
    gA[rows] = gA_I
    np.testing.assert_allclose(gA, g["grad_A"], rtol=1e-4, atol=1e-4)
    np.testing.assert_allclose(gB, g["grad_B"], rtol=1e-4, atol=1e-4)


def _prune(idx, m, n):
    rmask = np.zeros(m, bool); rmask[idx[0]] = True
    cmask = np.zeros(n, bool); cmask[idx[1]] = True
    rnew = np.cumsum(rmask) - 1
    cnew = np.cumsum(cmask) - 1
    return np.stack([rnew[idx[0]], cnew[idx[1]]]), rmask, cmask


def test_salsa_end_to_end(golden):
    g = golden("e2e_salsa")
    m, n, nb, it, seed = (int(g[k]) for k in ("m", "n", "num_blocks", "iters", "seed"))
    idx, rmask, cmask = _prune(g["S_index"], m, n)
    me, ne = int(rmask.sum()), int(cmask.sum())
    gr = torch.Generator().manual_seed(seed + 1)
    gc = torch.Generator().manual_seed(seed + 2)
    pr = [torch.randperm(me, generator=gr).numpy() for _ in range(it + 1)][1:]
    pc = [torch.randperm(ne, generator=gc).numpy() for _ in range(it + 1)][1:]
    A, B = orc.salsa_iterations(idx, g["S_value"], me, ne, g["A0"][rmask], g["B0"][cmask], nb, it,
                                0.7, float(g["lr"]), pr, pc)
    np.testing.assert_allclose(A, g["A"][rmask], rtol=1e-3, atol=1e-4)
    np.testing.assert_allclose(B, g["B"][cmask], rtol=1e-3, atol=1e-4)
    assert np.all(g["A"][~rmask] == 0) and np.all(g["B"][~cmask] == 0)


def test_gd_end_to_end(golden):
    g = golden("e2e_gd")
    m, n, nb, it, seed, bb = (int(g[k]) for k in ("m", "n", "num_blocks", "iters", "seed", "batch_blocks"))
    idx = g["S_index"]
    gb = torch.Generator().manual_seed(seed + 1)
    perm = torch.randperm(m, generator=gb).numpy()
    _, _, _, rows = orc.block_partition(perm, idx[0], nb)
    gl = torch.Generator().manual_seed(seed + 2)
    loader = torch.utils.data.DataLoader(list(range(nb)), batch_size=bb, shuffle=True, generator=gl,
                                         collate_fn=lambda b: b)
    batches = [[list(b) for b in loader] for _ in range(it)]
    A, B = orc.gd_epochs(idx, g["S_value"], g["A0"], g["B0"], rows, batches, it, float(g["lr"]))
    np.testing.assert_allclose(A, g["A"], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(B, g["B"], rtol=1e-4, atol=1e-5)
