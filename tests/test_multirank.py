"""The multi-GPU bench's host logic on two CPU ranks (gloo, 127.0.0.1).

Under torchrun each rank serves its own users with its own weight replica and
no per-step collective; only after the timed region do the ranks meet, to take
the slowest rank's span (the job's time) and gather every rank's per-user
latencies.  These tests run that logic in two spawned processes on the gloo
backend, so they need no GPU.
"""
import os
import socket
import sys
from pathlib import Path

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]
WORLD = 2


def free_port():
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def rank_main(rank, port, out):
    sys.path.insert(0, str(ROOT))
    import bench
    os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port))
    dist.init_process_group('gloo', rank=rank, world_size=WORLD)
    try:
        users = bench.rank_users(list(range(10)), rank, WORLD)
        # rank r's timed span and latencies; rank 1 is the slower one
        total = 100.0 + 50.0 * rank
        e2e = 120.0 + 10.0 * rank
        lat = [float(10 * rank + u) for u in users]
        e2e_lat = [x + 0.5 for x in lat]
        res = bench.combine_ranks(total, e2e, lat, e2e_lat, WORLD, 'cpu')
        torch.save({'users': users, 'res': res}, os.path.join(out, f'rank{rank}.pt'))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_ranks_deal_users_and_take_the_slowest_span(tmp_path):
    mp.start_processes(rank_main, args=(free_port(), str(tmp_path)), nprocs=WORLD, join=True, start_method='spawn')
    r0 = torch.load(tmp_path / 'rank0.pt')
    r1 = torch.load(tmp_path / 'rank1.pt')
    # users dealt round-robin: disjoint, together the whole list
    assert r0['users'] == [0, 2, 4, 6, 8] and r1['users'] == [1, 3, 5, 7, 9]
    for r in (r0, r1):  # every rank ends with the same job-level figures
        total, e2e, lat, e2e_lat = r['res']
        assert total == 150.0 and e2e == 130.0
        assert lat == [0.0, 2.0, 4.0, 6.0, 8.0, 11.0, 13.0, 15.0, 17.0, 19.0]
        assert e2e_lat == [x + 0.5 for x in lat]


def test_one_rank_keeps_its_own_figures():
    sys.path.insert(0, str(ROOT))
    import bench
    assert bench.rank_users([5, 6, 7], 0, 1) == [5, 6, 7]
    assert bench.combine_ranks(3.0, 4.0, [1.0], [2.0], 1, 'cpu') == (3.0, 4.0, [1.0], [2.0])
