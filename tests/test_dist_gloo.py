"""The multi-GPU bench's rank logic on CPU: two gloo ranks.

bench.py shards utterances across ranks (no collective on the token loop)
and uses torch.distributed only to time: a barrier around the timed region,
the max of the per-rank device times and the sum of the per-rank tokens.
"""
import os
import socket

import pytest
import torch.multiprocessing as mp

from conftest import ROOT


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank(rank, world, port, q):
    import sys
    sys.path.insert(0, str(ROOT))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    import bench
    d = bench.Dist(world, rank, backend="gloo", timeout_s=60)
    d.barrier()
    mx = d.max(10.0 + rank)      # per-rank "ms": the job time is the slowest rank's
    tot = d.sum(100.0 * (rank + 1))  # per-rank tokens: the job's tokens are the sum
    ids = bench.utterance_ids(rank, world, 64)             # one batch sharded (strong scaling)
    weak = bench.utterance_ids(rank, world, 4, weak=True)  # every rank its own batch
    d.barrier()
    d.close()
    q.put((rank, mx, tot, ids, weak))


def test_two_gloo_ranks_time_and_shard():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    res.sort()
    assert [r[1] for r in res] == [11.0, 11.0]
    assert [r[2] for r in res] == [300.0, 300.0]
    ids = res[0][3] + res[1][3]
    assert sorted(ids) == list(range(64)) and len(res[0][3]) == len(res[1][3]) == 32
    weak = res[0][4] + res[1][4]
    assert sorted(weak) == list(range(8)) and len(set(res[0][4]) & set(res[1][4])) == 0
