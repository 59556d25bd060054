"""Rank body for the multi-process tests of barracuda_b200.shard (gloo on
CPU, started with the `spawn` method).  Each scenario writes what rank 0
observed to a JSON file; failures are injected on the host only."""
import json
import os
import sys


def run(rank, world, port, scenario, out_path, total, seed):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    if root not in sys.path:
        sys.path.insert(0, root)
    from barracuda_b200.shard import Shard, ShardFailure, ShardGroup, job_digest
    from oracle import oracle as O

    result = {"rank": rank}
    try:
        group = ShardGroup("gloo", timeout=4.0)
    except ShardFailure as e:
        result.update(failure_rank=e.rank, failure=e.message, stage="rendezvous")
        _write(out_path, rank, result)
        return
    try:
        sh = Shard.of(total, world, rank)
        q = O.ntt_prime(31, 4096, 0)

        def local_digest():
            if scenario == "raise" and rank == 1:
                raise RuntimeError("injected failure on rank 1")
            if scenario == "exit" and rank == 1:
                os._exit(3)  # leaves without posting a status
            data = O.seeded_fill(sh.count, seed, sh.begin, q)
            return O.digest(data, sh.begin)

        d = group.step("digest", local_digest)
        rows = group.gather_u64([d, sh.begin, sh.count])
        result.update(rows=rows, job=job_digest(r[0] for r in rows))
    except ShardFailure as e:
        result.update(failure_rank=e.rank, failure=e.message, stage="step")
    except RuntimeError as e:
        result.update(raised=str(e))
    finally:
        if scenario == "ok":
            group.close()
    _write(out_path, rank, result)


def _write(out_path, rank, result):
    with open(f"{out_path}.{rank}", "w") as f:
        json.dump(result, f)
