"""The multi-GPU plumbing (mayfly_chess_b200/replicas.py) on the CPU: position shards, and the barrier and
max-over-ranks reduction over a world-size-2 gloo process group."""
import os
import socket

import pytest
import torch.multiprocessing as mp

from mayfly_chess_b200 import replicas


def test_shard_weak_and_strong():
    # weak: 1,024 per rank from rank * 1,024, wrapped when the set runs out
    assert replicas.shard(0, 8, 8192, per_rank=1024) == (0, 1024)
    assert replicas.shard(7, 8, 8192, per_rank=1024) == (7168, 1024)
    assert replicas.shard(1, 2, 8192, per_rank=4096) == (4096, 4096)
    assert replicas.shard(2, 4, 8192, per_rank=4096) == (0, 4096)
    # strong: the total split into contiguous shares covering it exactly once
    shares = [replicas.shard(r, 8, 8192, total=8192) for r in range(8)]
    assert shares[0] == (0, 1024) and shares[7] == (7168, 1024)
    covered = sorted(i for s, c in shares for i in range(s, s + c))
    assert covered == list(range(8192))
    with pytest.raises(ValueError):
        replicas.shard(0, 3, 8192, total=8192)
    with pytest.raises(ValueError):
        replicas.shard(0, 1, 100, per_rank=200)
    with pytest.raises(ValueError):
        replicas.shard(2, 2, 8192, per_rank=1)
    with pytest.raises(ValueError):
        replicas.shard(0, 2, 8192)


def test_single_process_needs_no_group():
    assert replicas.max_over_ranks(3.5) == 3.5
    replicas.barrier()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, out):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        r, w, lr = replicas.rank_env()
        replicas.barrier(dist)
        # each rank's "device time": the job's time is the slowest rank's
        t = replicas.max_over_ranks(10.0 + r * 5.5, dist)
        start, count = replicas.shard(r, w, 8192, total=8192)
        out.put((r, w, lr, t, start, count))
    finally:
        dist.destroy_process_group()


def test_two_rank_gloo_reduction():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert got == [(0, 2, 0, 15.5, 0, 4096), (1, 2, 1, 15.5, 4096, 4096)]


def _timed_step(rank, world):
    """What a bench rank does around its timed region: a barrier, its own work, the max over ranks."""
    import torch.distributed as dist
    replicas.barrier(dist)
    return replicas.max_over_ranks(1.0 + rank, dist)


def test_supervised_run_healthy():
    rep = replicas.run(_timed_step, 2, timeout_s=60, pg_timeout_s=20)
    assert rep.ok, rep.describe()
    assert rep.results == {0: 2.0, 1: 2.0}


@pytest.mark.parametrize("kind,why", [("raise", "raised RuntimeError: injected fault on rank 1"),
                                      ("exit", "exited with code 3"),
                                      ("hang", "no result within 20 s (killed)")])
def test_supervised_run_names_the_failed_rank(monkeypatch, kind, why):
    """A rank that raises, exits or stops answering (injected on the host) is named in the report, and the call
    returns within its deadline; the surviving rank's collective ends with an error (its process group times out
    or sees the peer gone) instead of waiting for ever."""
    import time
    monkeypatch.setenv(replicas.FAULT_ENV, f"1:{kind}")
    t0 = time.monotonic()
    rep = replicas.run(_timed_step, 2, timeout_s=20, pg_timeout_s=5)
    took = time.monotonic() - t0
    assert not rep.ok
    assert why in rep.failures.get(1, ""), rep.describe()
    assert 0 in rep.failures or 0 in rep.results
    assert took < 20 + 15, took
    assert f"rank 1: {why}" in rep.describe()


def test_inject_fault_spec():
    replicas.inject_fault(0, {})                                   # nothing set
    replicas.inject_fault(0, {replicas.FAULT_ENV: "1:raise"})      # another rank's fault
    with pytest.raises(RuntimeError, match="injected fault on rank 2"):
        replicas.inject_fault(2, {replicas.FAULT_ENV: "2:raise"})
    with pytest.raises(ValueError, match="unknown fault kind"):
        replicas.inject_fault(0, {replicas.FAULT_ENV: "0:melt"})
