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
