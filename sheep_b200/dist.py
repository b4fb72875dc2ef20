"""Multi-GPU plumbing for the bench: one process per GPU (torchrun), the
decode path run as independent replicas (batch-1 decode of one sequence does
not shard), times reduced as the max over ranks.

torch.distributed carries only the barrier and the max; no data of the decode
path crosses ranks.
"""
import os


def rank_info():
    """(world, rank, local_rank) from the torchrun environment."""
    return (int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")),
            int(os.environ.get("LOCAL_RANK", "0")))


def init(backend="nccl", timeout_s=300):
    """Initialise the process group when launched with more than one rank."""
    world, _, local = rank_info()
    if world <= 1:
        return None
    import datetime
    import torch
    import torch.distributed as dist
    if backend == "nccl":
        torch.cuda.set_device(local)
    dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s))
    return dist


def max_over_ranks(dist, value, device="cuda"):
    if dist is None:
        return float(value)
    import torch
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def replica_throughput(steps, seconds_max, world):
    """Whole-job tokens/s of `world` replicas that each ran `steps` tokens,
    the slowest taking `seconds_max` (weak scaling)."""
    return world * steps / seconds_max
