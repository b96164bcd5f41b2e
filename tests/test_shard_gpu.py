"""Sharded solvers on two GPUs (two NCCL ranks, sumac_b200/shard.py) against the reference's own
runs (tests/golden/e2e_salsa.npz, e2e_gd.npz): the same factors and history as the single-GPU
paths. Skipped when fewer than two GPUs are visible."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from tests.conftest import load_golden
from tests.helpers import rel_err

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q, method="salsa"):
    try:
        import torch.distributed as dist
        from sumac_b200 import SumacConfig, SumacMethod, sumac_factorize
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world,
                                device_id=torch.device("cuda", rank))
        g = load_golden("e2e_" + method)
        extra = (dict(eval_interval=1) if method == "salsa" else
                 dict(eval_interval=2, batch_blocks=int(g["batch_blocks"]), shuffle_blocks=True))
        cfg = SumacConfig(method=SumacMethod.SALSA if method == "salsa" else SumacMethod.GD,
                          rank=int(g["rank"]), max_iterations=int(g["iters"]),
                          num_blocks=int(g["num_blocks"]), seed=int(g["seed"]),
                          learning_rate=float(g["lr"]), verbose=False, perm_device="cpu",
                          device=f"cuda:{rank}", **extra)
        dev = torch.device("cuda", rank)
        A, B, hist = sumac_factorize(S_index=torch.from_numpy(g["S_index"]).to(dev),
                                     S_value=torch.from_numpy(g["S_value"]).to(dev),
                                     shape=(int(g["m"]), int(g["n"])),
                                     A_init=torch.from_numpy(g["A0"]).to(dev),
                                     B_init=torch.from_numpy(g["B0"]).to(dev), config=cfg)
        dist.destroy_process_group()
        q.put((rank, A.cpu().numpy(), B.cpu().numpy(), hist, None))
    except Exception as e:  # reported to the parent instead of hanging it
        q.put((rank, None, None, None, repr(e)))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("method", ["salsa", "gd"])
def test_sharded_solver_matches_reference_run(method):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, method)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    g = load_golden("e2e_" + method)
    for rank, A, B, hist, err in res:
        assert err is None, (rank, err)
        assert rel_err(A, g["A"]) < 1e-4
        assert rel_err(B, g["B"]) < 1e-4
        for key in ("cost", "rmse", "jacc"):
            np.testing.assert_allclose(hist[key], g[key], rtol=1e-4)
    # every rank returns the same whole factors
    assert np.array_equal(res[0][1], res[1][1]) and np.array_equal(res[0][2], res[1][2])
