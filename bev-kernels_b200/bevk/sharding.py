"""Batch x camera sharding for multi-GPU runs of the deformable-sampling path.

The path shards trivially: a DCN output pixel depends only on its own image and
an MSDA query of camera b reads only value[b].  Work is split into contiguous
blocks of images, one block per rank, with no collective on the data path;
every rank regenerates or loads its own block, so no input is scattered.
"""
from __future__ import annotations


def shard_range(n_items: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous [begin, end) block of `n_items` owned by `rank` of `world`.

    Blocks differ in size by at most one item; ranks beyond n_items get an empty
    block.
    """
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    base, extra = divmod(n_items, world)
    begin = rank * base + min(rank, extra)
    return begin, begin + base + (1 if rank < extra else 0)


def image_seed(seed: int, image: int, salt: int = 0) -> int:
    """Generator seed of global image `image`: a rank derives its shard's data
    from (seed, global image index) alone, independent of the world size."""
    return (seed * 1_000_003 + image * 101 + salt) & 0x7FFFFFFFFFFFFFFF
