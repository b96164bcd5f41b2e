"""Host logic of the row-sharded SALSA (sumac_b200/shard.py) on two gloo ranks on the CPU:
shard ranges, the split of S by updated row, the exact allreduce assembly of block rows and the
all-gather of a sharded factor."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from sumac_b200.shard import assemble_rows, gather_rows, shard_range, split_direction


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        g = torch.Generator().manual_seed(0)
        m, Dp = 37, 16
        F = torch.randn(m, Dp, generator=g)
        lo, hi = shard_range(m, rank, world)
        rows = torch.randperm(m, generator=g)[:11]
        out = torch.full((rows.numel(), Dp), float("nan"))
        assemble_rows(F[lo:hi].clone(), lo, hi, rows, out)
        ok_assemble = torch.equal(out, F[rows])
        whole = gather_rows(F[lo:hi].clone(), m)
        ok_gather = torch.equal(whole, F)
        dist.destroy_process_group()
        q.put((rank, ok_assemble, ok_gather))
    except Exception as e:  # reported to the parent instead of hanging it
        q.put((rank, repr(e), None))


def test_shard_ranges_cover_rows_once():
    for total in (1, 7, 100, 139255):
        for world in (1, 2, 3, 8):
            if total < world:
                continue
            rs = [shard_range(total, r, world) for r in range(world)]
            assert rs[0][0] == 0 and rs[-1][1] == total
            assert all(rs[r][1] == rs[r + 1][0] for r in range(world - 1))
            assert max(h - l for l, h in rs) - min(h - l for l, h in rs) <= 1


def test_split_direction_partitions_entries():
    g = torch.Generator().manual_seed(1)
    i = torch.randint(0, 50, (400,), generator=g)
    j = torch.randint(0, 30, (400,), generator=g)
    for world in (2, 3):
        seen = torch.zeros(400, dtype=torch.int32)
        for r in range(world):
            seen += split_direction(i, j, *shard_range(30, r, world)).int()
        assert torch.all(seen == 1)


def test_assemble_and_gather_two_gloo_ranks():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, a, b in res:
        assert a is True and b is True, (rank, a, b)


def test_gd_subblocks_partition_every_position_once():
    from sumac_b200.shard import subblock_bounds, virtual_positions
    for m, nb, world in [(1000, 7, 2), (8131 * 3 + 5, 4, 8), (50, 10, 3), (97, 1, 4)]:
        bs = (m + nb - 1) // nb
        bsub = (bs + world - 1) // world
        pos = torch.arange(m)
        owner = torch.full((m,), -1)
        for r in range(world):
            v = virtual_positions(pos, m, nb, r, world)
            own = v >= 0
            assert torch.all(owner[own] == -1)
            owner[own] = r
            vv = v[own]
            assert vv.unique().numel() == vv.numel() and int(vv.max()) < nb * bsub
            # a position keeps its block, and its slot within the sub-block
            k = pos[own] // bs
            assert torch.equal(vv // bsub, k)
            lo = torch.tensor([subblock_bounds(m, nb, int(kk), r, world)[0] for kk in k])
            assert torch.equal(vv % bsub, pos[own] - k * bs - lo)
        assert torch.all(owner >= 0)


def _gd_worker(rank, world, port, q):
    """Each rank forms the oracle's gradient of its sub-blocks only (its rows of the block, their
    entries of S), then combine_block_grads completes the step's gradients; they must equal the
    oracle's gradient of the whole batch of blocks."""
    try:
        import numpy as np

        from oracle import sumac_oracle as orc
        from sumac_b200.shard import combine_block_grads, subblock_bounds
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        rng = np.random.default_rng(0)
        m, n, d, nb = 41, 30, 4, 3
        A = rng.standard_normal((m, d))
        B = rng.standard_normal((n, d))
        keys = rng.choice(m * n, 300, replace=False)
        si, sj, sv = keys // n, keys % n, 0.1 + rng.random(300)
        perm = rng.permutation(m)
        bs = (m + nb - 1) // nb
        batch = [0, 2]
        gA = torch.zeros((m, d), dtype=torch.float64)
        gB = torch.zeros((n, d), dtype=torch.float64)
        gA_ref = np.zeros((m, d))
        gB_ref = np.zeros((n, d))
        block_rows = []
        for k in batch:
            full = perm[k * bs:min(m, (k + 1) * bs)]
            block_rows.append(torch.from_numpy(full))
            lo, hi = subblock_bounds(m, nb, k, rank, world)
            for rows, acc_a, acc_b in ((full[lo:hi], gA, gB), (full, None, None)):
                pos = {r: t for t, r in enumerate(rows)}
                sel = [e for e in range(300) if si[e] in pos]
                li = [pos[si[e]] for e in sel]
                _, g_ai, g_b = orc.gd_block_grad(A[rows], B, li, sj[sel], sv[sel])
                if acc_a is not None:
                    acc_a[torch.from_numpy(rows)] += torch.from_numpy(g_ai)
                    acc_b += torch.from_numpy(g_b)
                else:
                    gA_ref[rows] += g_ai
                    gB_ref += g_b
        combine_block_grads(gA, gB, block_rows, torch.zeros((bs, d), dtype=torch.float64))
        ok = bool(np.allclose(gA.numpy(), gA_ref, rtol=1e-12, atol=1e-12) and
                  np.allclose(gB.numpy(), gB_ref, rtol=1e-12, atol=1e-12))
        dist.destroy_process_group()
        q.put((rank, ok, None))
    except Exception as e:  # reported to the parent instead of hanging it
        q.put((rank, repr(e), None))


def test_sharded_gd_gradient_combination_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gd_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, ok, _ in results:
        assert ok is True, (rank, ok)
