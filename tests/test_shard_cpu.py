"""Host-side logic of member sharding, on CPU with the gloo backend (world size 2)."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle.philox import permutation_keys
from tabpack_b200.shard import allreduce_sum_, gather_members, member_ranges


def test_member_ranges_cover_members_in_order():
    for n, w in [(10, 3), (8, 8), (512, 8), (7, 2)]:
        r = member_ranges(n, w)
        assert r[0][0] == 0 and r[-1][1] == n
        assert all(r[k][1] == r[k + 1][0] for k in range(w - 1))
        assert max(b - a for a, b in r) - min(b - a for a, b in r) <= 1
    cost = [float(c) for c in np.random.default_rng(0).integers(1, 100, 64)]
    r = member_ranges(64, 4, cost)
    loads = [sum(cost[a:b]) for a, b in r]
    assert max(loads) - min(loads) <= max(cost)


@pytest.mark.parametrize('n,world,cost', [
    (4, 4, [10.0, 1.0, 1.0, 1.0]),
    (8, 4, [100.0] + [1.0] * 7),
    (8, 4, [1.0] * 7 + [100.0]),
    (9, 8, [1.0, 1.0, 1.0, 1.0, 50.0, 1.0, 1.0, 1.0, 1.0]),
    (512, 8, [1e6] + [1.0] * 511),
])
def test_member_ranges_skewed_cost_leaves_no_rank_empty(n, world, cost):
    r = member_ranges(n, world, cost)
    assert r[0][0] == 0 and r[-1][1] == n
    assert all(r[k][1] == r[k + 1][0] for k in range(world - 1))
    assert all(b > a for a, b in r), r


def test_member_ranges_fewer_members_than_ranks_raises_on_every_rank():
    from tabpack_b200.training import PackTrainer

    r = member_ranges(2, 4, [1.0, 5.0])
    assert r[0][0] == 0 and r[-1][1] == 2 and sum(b - a for a, b in r) == 2
    # the check runs on the ranges every rank computes alike, before any collective
    with pytest.raises(ValueError, match='every rank needs at least one member'):
        PackTrainer._check_ranges(r)


def test_permutation_keys_depend_only_on_global_member():
    full = permutation_keys(seed=123, epoch=4, members=np.arange(10), n_rows=257)
    part = permutation_keys(seed=123, epoch=4, members=np.arange(6, 10), n_rows=257)
    assert np.array_equal(full[6:], part)
    assert full.min() >= 0
    # different epochs reshuffle
    assert not np.array_equal(full, permutation_keys(seed=123, epoch=5, members=np.arange(10), n_rows=257))


def _free_port():
    s = socket.socket()
    s.bind(('127.0.0.1', 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    os.environ['MASTER_ADDR'] = '127.0.0.1'
    os.environ['MASTER_PORT'] = str(port)
    dist.init_process_group('gloo', rank=rank, world_size=world)
    try:
        ranges = member_ranges(5, world)  # uneven: 3 + 2 members
        lo, hi = ranges[rank]
        counts = [b - a for a, b in ranges]
        local = torch.stack([torch.full((4, 3), float(m)) for m in range(lo, hi)])
        allm = gather_members(local, counts)
        s = allreduce_sum_(torch.tensor([float(rank + 1)]))
        q.put((rank, allm[:, 0, 0].tolist(), float(s)))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(120)
def test_gather_members_gloo_world2():
    ctx = mp.get_context('spawn')
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=90) for _ in range(2)]
    for p in procs:
        p.join(timeout=30)
        assert p.exitcode == 0
    for rank, members, s in res:
        assert members == [0.0, 1.0, 2.0, 3.0, 4.0]
        assert s == 3.0
