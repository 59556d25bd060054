"""CPU tests of the multi-GPU split (barracuda_b200.shard): the shard ranges
cover every unit once, per-shard digests add up to the digest of the whole
job, and a failed, exited or missing rank reaches its peers as
ShardFailure within the deadline instead of a hang.  The multi-rank cases
run as gloo process groups of world size 2 on 127.0.0.1; failures are
injected on the host (an exception, an exit, a rank that never starts)."""
import json
import multiprocessing as mp
import os
import socket
import time

import numpy as np
import pytest

from barracuda_b200.shard import Shard, job_digest
from oracle import oracle as O
from tests import shard_worker


@pytest.mark.parametrize("total,world", [(128, 1), (128, 2), (128, 8), (48, 3), (5, 8), (0, 4)])
def test_shard_ranges_cover_every_unit_once(total, world):
    shards = [Shard.of(total, world, r) for r in range(world)]
    pos = 0
    for s in shards:
        assert s.begin == pos
        pos += s.count
    assert pos == total
    sizes = [s.count for s in shards]
    assert max(sizes) - min(sizes) <= 1


def test_shard_digests_add_up_to_the_job_digest():
    q = O.ntt_prime(31, 4096, 0)
    total = 10_000
    whole = O.seeded_fill(total, 9, 0, q)
    for world in (1, 2, 3, 8):
        parts = []
        for r in range(world):
            s = Shard.of(total, world, r)
            part = O.seeded_fill(s.count, 9, s.begin, q)
            assert (part == whole[s.begin:s.begin + s.count]).all()  # inputs from global indices
            parts.append(O.digest(part, s.begin))
        assert job_digest(parts) == O.digest(whole, 0)
    assert O.digest(whole, 0) != O.digest(whole[::-1].copy(), 0)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(tmp_path, scenario, ranks=(0, 1), world=2, total=4096, seed=3, deadline=90):
    ctx = mp.get_context("spawn")
    port = _free_port()
    out = str(tmp_path / scenario)
    procs = [ctx.Process(target=shard_worker.run, args=(r, world, port, scenario, out, total, seed))
             for r in ranks]
    for p in procs:
        p.start()
    t0 = time.time()
    for p in procs:
        p.join(max(1.0, deadline - (time.time() - t0)))
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
        p.join()
    assert not alive, f"{scenario}: ranks still running after {deadline} s (hang)"
    res = {}
    for r in ranks:
        path = f"{out}.{r}"
        if os.path.exists(path):
            with open(path) as f:
                res[r] = json.load(f)
    return res, time.time() - t0


def test_two_ranks_gather_shard_digests(tmp_path):
    total, seed = 4096, 3
    res, _ = _run(tmp_path, "ok", total=total, seed=seed)
    q = O.ntt_prime(31, 4096, 0)
    want = O.digest(O.seeded_fill(total, seed, 0, q), 0)
    for r in (0, 1):
        rows = res[r]["rows"]
        assert [row[1:] for row in rows] == [[0, 2048], [2048, 2048]]
        assert res[r]["job"] == want


def test_rank_that_raises_reaches_its_peer(tmp_path):
    res, _ = _run(tmp_path, "raise")
    assert res[0]["failure_rank"] == 1
    assert "injected failure on rank 1" in res[0]["failure"]
    assert "injected" in res[1]["raised"]


def test_rank_that_exits_is_detected_by_deadline(tmp_path):
    res, took = _run(tmp_path, "exit")
    assert res[0]["failure_rank"] == 1 and "no status" in res[0]["failure"]
    assert 1 not in res
    assert took < 60


def test_rank_that_never_joins_fails_the_rendezvous(tmp_path):
    res, took = _run(tmp_path, "nojoin", ranks=(0,))
    assert res[0]["stage"] == "rendezvous"
    assert took < 60
