"""Multi-GPU plumbing: one process per GPU, torch.distributed for rendezvous,
the max-over-ranks timing reduction, and the hand-over of the NCCL id that
row-sharded decode states share.

The default decode shards by sequence (independent replicas of the model,
each rank decoding its own sequences): no data-path collective. A row-sharded
state (State.shard) splits every GEMV's rows over the ranks and all-gathers
each output through the library's own NCCL communicator.
"""
import os


def env_rank():
    return int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")), \
        int(os.environ.get("LOCAL_RANK", "0"))


def shard_range(n, rank, world):
    """contiguous [lo, hi) share of n units for rank (sizes differ by at most 1)."""
    base, extra = divmod(n, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def init(backend=None, timeout_s=120):
    """initialise the process group from torchrun's environment (no-op at world 1)."""
    import datetime
    import torch.distributed as dist
    rank, world, _ = env_rank()
    if world <= 1 or dist.is_initialized():
        return rank, world
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    dist.init_process_group(backend=backend or "nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))
    return rank, world


def max_over_ranks(value, device=None):
    """the maximum of a float over all ranks (the value itself at world 1)."""
    import torch
    import torch.distributed as dist
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(value, device=None):
    import torch
    import torch.distributed as dist
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def barrier():
    import torch.distributed as dist
    if dist.is_initialized():
        dist.barrier()


def finish():
    import torch.distributed as dist
    if dist.is_initialized():
        dist.destroy_process_group()


def share_from_rank0(make):
    """the value make() returns on rank 0, on every rank (picklable)"""
    import torch.distributed as dist
    rank, world, _ = env_rank()
    if world <= 1 or not dist.is_initialized():
        return make()
    box = [make() if rank == 0 else None]
    dist.broadcast_object_list(box, src=0)
    return box[0]

