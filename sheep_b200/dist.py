"""Multi-GPU plumbing for the bench: one process per GPU (torchrun), the
decode path run as independent replicas (batch-1 decode of one sequence does
not shard), times reduced as the max over ranks; and the host side of the
expert-parallel MoE layer (sb_moe_open_ep): the NCCL id every rank must share
and the experts each rank holds.

torch.distributed carries only the barrier, the max and the id; the MoE layer's
data crosses ranks in the library's own NCCL all-reduce.
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


def expert_range(n_expert, world, rank):
    """The experts rank `rank` of `world` holds: [lo, hi) (as sb_moe_open_ep)."""
    return n_expert * rank // world, n_expert * (rank + 1) // world


def share_nccl_id(dist, device="cuda"):
    """The 128-byte NCCL id made by rank 0 (sb_nccl_unique_id), broadcast to every rank."""
    import torch
    import sheep_b200
    _, rank, _ = rank_info()
    t = torch.zeros(128, dtype=torch.uint8, device=device)
    if rank == 0:
        t.copy_(torch.frombuffer(bytearray(sheep_b200.nccl_unique_id()), dtype=torch.uint8))
    if dist is not None:
        dist.broadcast(t, src=0)
    return bytes(t.cpu().numpy().tobytes())
