"""Data-parallel plumbing for the batched decoder: one replica per GPU, the
requests partitioned round-robin across ranks, and the run statistics
reduced once at the end.  There is no collective on the per-step path (the
requests of different ranks never interact, as in the reference, which
serves them independently: surface/mod.rs:96-106)."""
import torch
import torch.distributed as dist


def partition(n_requests, rank, world):
    """Request indices that rank `rank` of `world` serves (i mod world)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    return [i for i in range(n_requests) if i % world == rank]


def reduce_stats(stats, device="cpu"):
    """stats: {name: (value, "sum" | "max")} with the same names in the same
    order on every rank.  Returns {name: reduced value}.  Always two
    collectives (one SUM, one MAX), so every rank takes the same steps."""
    for name, (_, op) in stats.items():
        if op not in ("sum", "max"):
            raise ValueError(f"{name}: unknown reduction {op!r}")
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return {k: float(v) for k, (v, _) in stats.items()}
    names = list(stats)
    sums = torch.tensor([float(stats[k][0]) if stats[k][1] == "sum" else 0.0 for k in names],
                        dtype=torch.float64, device=device)
    maxs = torch.tensor([float(stats[k][0]) if stats[k][1] == "max" else float("-inf") for k in names],
                        dtype=torch.float64, device=device)
    dist.all_reduce(sums, op=dist.ReduceOp.SUM)
    dist.all_reduce(maxs, op=dist.ReduceOp.MAX)
    return {k: (sums[i].item() if stats[k][1] == "sum" else maxs[i].item()) for i, k in enumerate(names)}
