"""Multi-GPU partitioning on the CPU: every unit is a contiguous sub-problem
of the unchanged ABI, units cover the output exactly once, and a 2-rank gloo
job that computes its shard through those offsets (with the oracle standing in
for the device) reassembles the full result; timing reduces to the max over
ranks."""
import dataclasses
import math
import os
import socket

import numpy as np
import pytest

from groupconv_atlas_b200.api import Shape, inputs
from groupconv_atlas_b200 import shard
from oracle import oracle as orc


@pytest.mark.parametrize('n,groups,world', [(32, 256, 1), (32, 256, 2), (1024, 32, 8), (7, 4, 3),
                                            (1, 8, 8), (2, 4, 8), (3, 6, 4), (1, 32, 2)])
def test_units_cover_output_exactly_once(n, groups, world):
    s = Shape(n=n, cin=groups * 2, cout=groups * 2, h=5, w=6, groups=groups)
    seen = np.zeros((s.n, s.cout), np.int32)
    per_rank = []
    for rank in range(world):
        units = shard.units_for_rank(s, world, rank)
        per_rank.append(sum(u.images() * (u.c1 - u.c0) for u in units))
        for u in units:
            sub = u.shape(s)
            assert sub.cin % sub.groups == 0 and sub.cin // sub.groups == s.cpg
            seen[u.n0:u.n1, u.c0:u.c1] += 1
            ox, ow, oy = u.offsets(s)
            assert ox + math.prod(sub.input) <= math.prod(s.input)
            assert oy + math.prod(sub.output) <= math.prod(s.output)
            assert ow + math.prod(sub.weight) <= math.prod(s.weight)
    assert (seen == 1).all()
    # balanced: ranks differ by at most one unit's worth of work
    assert max(per_rank) - min(per_rank) <= max(s.cout, (s.cout // min(world, s.groups)) + s.cout)


def _free_port():
    with socket.socket() as sock:
        sock.bind(('127.0.0.1', 0))
        return sock.getsockname()[1]


def _rank_main(rank, world, port, shape_dict, result_path):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port))
    dist.init_process_group('gloo', rank=rank, world_size=world)
    try:
        s = Shape(**shape_dict)
        x, w = inputs(s, 11)
        y = np.zeros(s.output, np.float32)
        for u in shard.units_for_rank(s, world, rank):
            sub = u.shape(s)
            ox, ow, oy = u.offsets(s)
            xs = x.reshape(-1)[ox:ox + math.prod(sub.input)].reshape(sub.input)
            ws = w.reshape(-1)[ow:ow + math.prod(sub.weight)].reshape(sub.weight)
            ys = orc.conv_f32_serial(sub, xs, ws)
            y.reshape(-1)[oy:oy + ys.size] = ys.reshape(-1)
        gathered = [None] * world
        dist.all_gather_object(gathered, y)
        slowest = shard.max_over_ranks(float(rank + 1) * 1.5)
        total = shard.sum_over_ranks(1.0)
        if rank == 0:
            full = sum(gathered)
            np.save(result_path, full)
            np.save(str(result_path) + '.timing.npy', np.array([slowest, total]))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize('shape_dict', [
    dict(n=4, cin=8, cout=8, h=9, w=11, groups=4),    # batch sharding
    dict(n=1, cin=8, cout=8, h=9, w=11, groups=8),    # group-block sharding (N < world)
])
def test_gloo_two_ranks_reassemble(tmp_path, shape_dict):
    import torch.multiprocessing as mp
    world, port = 2, _free_port()
    out = tmp_path / 'y.npy'
    mp.start_processes(_rank_main, args=(world, port, shape_dict, str(out)), nprocs=world,
                       start_method='spawn', join=True)
    s = Shape(**shape_dict)
    x, w = inputs(s, 11)
    full = np.load(out)
    assert np.array_equal(full, orc.conv_f32_serial(s, x, w))
    slowest, total = np.load(str(out) + '.timing.npy')
    assert slowest == 3.0 and total == 2.0
