"""Several GPUs: one independent evaluator per GPU, the leaf batch split by position.

The search's batch shards by position with no exchange between the shards (the reference runs one evaluation
server per card, mayfly/chess/selfplay_remote.py:505-520), so a multi-GPU run needs no data collective: each
rank evaluates its own positions. What the ranks do share is plumbing: which positions each takes, a barrier
around a timed region, and the max over ranks of a device time (a job is as slow as its slowest rank). Those are
here, for torch.distributed process groups of any backend (NCCL on the GPUs; gloo in the CPU tests).
"""
import os


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
