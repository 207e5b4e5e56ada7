"""Batch sharding across GPUs (one process per GPU, no data-path collective).

Every benchmark configuration is independent along its batch dimension (MLP rows,
attention batch elements, conv images, encoder sequences): rank r of W processes
the contiguous block shard_range(B, r, W).
"""


def shard_range(total, rank, world):
    """[start, stop) of rank's contiguous block; the first total % world ranks get one extra."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of world {world}")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)
