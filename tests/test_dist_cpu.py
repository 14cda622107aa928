"""Box partition logic on CPU: two gloo ranks (world size 2, 127.0.0.1) stand in for two GPUs.

Inferences are independent, so ranks share no data: each draws a disjoint block of seeds, and the only
cross-rank steps are the max of the timed intervals and the x0-digest agreement check."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from vela_b200.dist import seed_block, golden_seeds, max_over_ranks, digests_agree


def _port():
    s = socket.socket(); s.bind(("127.0.0.1", 0)); p = s.getsockname()[1]; s.close()
    return p


def _worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        seeds = np.concatenate([seed_block(rank, l, s, 8) for l in range(2) for s in range(3)])
        t = max_over_ranks(1.5 + rank)
        same = digests_agree(bytes(range(32)))
        diff = digests_agree(bytes([rank]) * 32)
        q.put((rank, seeds, t, same, diff))
    finally:
        dist.destroy_process_group()


def test_two_ranks_partition_and_reduce():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict((r[0], r[1:]) for r in (q.get(timeout=120) for _ in ps))
    for p in ps:
        p.join(60)
        assert p.exitcode == 0
    s0, s1 = res[0][0], res[1][0]
    rows = {bytes(r) for r in np.concatenate([s0, s1])}
    assert len(rows) == len(s0) + len(s1), "seed blocks overlap across ranks / lanes / steps"
    assert res[0][1] == res[1][1] == 2.5, "max over ranks"
    assert res[0][2] and res[1][2], "equal digests agree"
    assert not res[0][3] and not res[1][3], "different digests must disagree on every rank"


def test_single_process_helpers():
    assert max_over_ranks(3.25) == 3.25 and digests_agree(b"x" * 32)
    a = seed_block(0, 0, 0, 8)
    assert a.shape == (8, 32) and a.dtype == np.uint8
    assert np.array_equal(a, seed_block(0, 0, 0, 8)), "deterministic"
    assert not np.array_equal(a, seed_block(1, 0, 0, 8))


def test_golden_seeds_are_the_fixture_seeds(golden):
    e = golden("engine")
    assert np.array_equal(golden_seeds(len(e["seeds"])), e["seeds"])
