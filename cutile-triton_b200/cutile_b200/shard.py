"""Data-parallel partition of the workloads over ranks (one process
per GPU). Every unit is independent — vadd elements, rowsum/softmax/
layernorm rows, GEMM row blocks, batched-GEMM batches, attention
(batch, head) pairs — so ranks exchange nothing on the data path.
"""


def shard_range(total, rank, world, align=1):
    """Contiguous [lo, hi) slice of `total` units for `rank` of `world`,
    boundaries rounded to multiples of `align` (the last rank takes the rest)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad rank/world")
    units = (total + align - 1) // align
    lo = (units * rank) // world * align
    hi = (units * (rank + 1)) // world * align
    return min(lo, total), min(hi, total)


def weak_offset(units_per_rank, rank):
    """Weak scaling: rank r processes units [r*U, (r+1)*U) of an N-times larger
    job, so per-GPU work stays fixed as N grows; used as the seed counter
    offset so every rank's synthetic inputs are distinct and reproducible."""
    return units_per_rank * rank


def gather_shards(local, group=None):
    """Optional final gather: every rank's equal-sized shard (dim 0) of a
    result, concatenated in rank order on every rank. Not part of the data
    path; over NCCL it moves the shards across NVLink/NVSwitch, over gloo
    it runs on host tensors (used by the CPU tests)."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    parts = [torch.empty_like(local) for _ in range(world)]
    dist.all_gather(parts, local.contiguous(), group=group)
    return torch.cat(parts, dim=0)
