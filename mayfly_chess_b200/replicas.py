"""Several GPUs: one independent evaluator per GPU, the leaf batch split by position.

The search's batch shards by position with no exchange between the shards (the reference runs one evaluation
server per card, mayfly/chess/selfplay_remote.py:505-520), so a multi-GPU run needs no data collective: each
rank evaluates its own positions. What the ranks do share is plumbing: which positions each takes, a barrier
around a timed region, and the max over ranks of a device time (a job is as slow as its slowest rank). Those are
here, for torch.distributed process groups of any backend (NCCL on the GPUs; gloo in the CPU tests).
"""
import os
import queue as _queue
import socket
import time
import traceback


def rank_env():
    """(rank, world size, local rank) from the torchrun environment (1 process, rank 0 without one)."""
    r = int(os.environ.get("RANK", "0"))
    w = int(os.environ.get("WORLD_SIZE", "1"))
    lr = int(os.environ.get("LOCAL_RANK", str(r)))
    return r, w, lr


def shard(rank, world, n_positions, per_rank=None, total=None):
    """(start, count) of this rank's positions in a set of n_positions.

    total: strong scaling, `total` positions split evenly over the ranks (rank r takes the r-th contiguous
    share); per_rank: weak scaling, `per_rank` positions each, rank r starting at r * per_rank, wrapped to the
    start of the set when the set is too small for every rank to have its own."""
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside 0..{world - 1}")
    if (total is None) == (per_rank is None):
        raise ValueError("give exactly one of per_rank and total")
    if total is not None:
        if total % world:
            raise ValueError(f"{total} positions do not split over {world} ranks")
        count = total // world
        start = rank * count
        if start + count > n_positions:
            raise ValueError(f"{total} positions but the set holds {n_positions}")
        return start, count
    if per_rank > n_positions:
        raise ValueError(f"{per_rank} positions per rank but the set holds {n_positions}")
    start = (rank * per_rank) % n_positions
    return (start if start + per_rank <= n_positions else 0), per_rank


def barrier(dist=None, device_sync=None):
    """A barrier over the default process group (when there is one), then the device synchronised."""
    if dist is not None and dist.is_initialized() and dist.get_world_size() > 1:
        dist.barrier()
    if device_sync is not None:
        device_sync()


def max_over_ranks(x, dist=None, device="cpu"):
    """The largest x over the ranks of the default process group (x itself without one)."""
    if dist is None or not dist.is_initialized() or dist.get_world_size() == 1:
        return float(x)
    import torch
    t = torch.tensor([float(x)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ------------------------------------------------------------------------------------------------ supervised runs
# A job of N independent evaluators is only as good as its slowest rank, and a rank can fail on its own: raise,
# exit, or stop answering. run() launches one process per rank, gives each a process group whose collectives
# time out (so the surviving ranks of a broken job end with an error instead of waiting forever), and watches
# them from the parent with a deadline: a rank that raised, exited without a result or is still running at the
# deadline is named in the report, and the parent never waits past the deadline (it kills its own children that
# are left). This is the role of the reference's watch over its evaluation servers
# (mayfly/chess/selfplay_remote.py:522-529: a server that dies is reported, not waited for).
#
# Faults are injected on the host, before a rank's work: MAYFLY_REPLICA_FAULT="<rank>:<kind>" with kind "raise"
# (an exception), "exit" (os._exit(3)) or "hang" (sleeps past any deadline). Nothing is injected on a GPU.

FAULT_ENV = "MAYFLY_REPLICA_FAULT"


class RunReport:
    """results: {rank: what the rank's function returned}; failures: {rank: why it has no result}."""

    def __init__(self, world, results, failures, seconds):
        self.world, self.results, self.failures, self.seconds = world, results, failures, seconds

    @property
    def ok(self):
        return not self.failures and len(self.results) == self.world

    def describe(self):
        if self.ok:
            return f"{self.world} ranks ok in {self.seconds:.1f} s"
        return "; ".join(f"rank {r}: {why}" for r, why in sorted(self.failures.items()))


def inject_fault(rank, env=None):
    """Applies MAYFLY_REPLICA_FAULT to this rank (a no-op unless it names this rank)."""
    spec = (env if env is not None else os.environ).get(FAULT_ENV, "")
    if not spec:
        return
    who, _, kind = spec.partition(":")
    if int(who) != rank:
        return
    if kind == "raise":
        raise RuntimeError(f"injected fault on rank {rank}")
    if kind == "exit":
        os._exit(3)
    if kind == "hang":
        time.sleep(10 ** 6)
    raise ValueError(f"{FAULT_ENV}: unknown fault kind {kind!r}")


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(fn, rank, world, port, backend, pg_timeout_s, out, args):
    import torch.distributed as dist
    from datetime import timedelta
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    try:
        dist.init_process_group(backend, rank=rank, world_size=world, timeout=timedelta(seconds=pg_timeout_s))
        try:
            inject_fault(rank)
            out.put(("ok", rank, fn(rank, world, *args)))
        finally:
            dist.destroy_process_group()
    except BaseException as e:     # noqa: BLE001 - every failure goes back to the parent as text
        last = traceback.format_exception_only(type(e), e)[-1].strip()
        out.put(("error", rank, last[:500]))


def run(fn, world, timeout_s=120.0, backend="gloo", pg_timeout_s=30.0, args=()):
    """Runs fn(rank, world, *args) on `world` spawned processes joined by a `backend` process group and returns a
    RunReport within about timeout_s seconds whatever the ranks do. fn must be picklable (a module-level
    function); what it returns comes back in report.results."""
    import multiprocessing as mp
    ctx = mp.get_context("spawn")    # never fork a process that may hold a CUDA context
    out = ctx.Queue()
    port = _free_port()
    procs = {r: ctx.Process(target=_rank_main, args=(fn, r, world, port, backend, pg_timeout_s, out, args),
                            daemon=True) for r in range(world)}
    t0 = time.monotonic()
    for p in procs.values():
        p.start()
    results, failures = {}, {}
    deadline = t0 + timeout_s
    exited_at = {}
    while len(results) + len(failures) < world:
        try:
            kind, rank, val = out.get(timeout=0.2)
            if kind == "ok":
                results[rank] = val
            else:
                failures[rank] = f"raised {val}"
            continue
        except _queue.Empty:
            pass
        now = time.monotonic()
        for r, p in procs.items():
            if r in results or r in failures or p.is_alive():
                continue
            # a rank that exited puts its message before it exits: give the queue a moment to deliver it
            exited_at.setdefault(r, now)
            if now - exited_at[r] > 2.0:
                failures[r] = f"exited with code {p.exitcode} and no result"
        if now > deadline:
            for r, p in procs.items():
                if r not in results and r not in failures:
                    failures[r] = f"no result within {timeout_s:.0f} s (killed)"
            break
    for p in procs.values():
        if p.is_alive():
            p.kill()
        p.join(timeout=5)
    return RunReport(world, results, failures, time.monotonic() - t0)
