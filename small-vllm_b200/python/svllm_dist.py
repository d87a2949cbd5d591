"""Token-row sharding across the GPUs of one node.

Every layer op here is independent per token row, so a batch of T rows splits into contiguous,
balanced ranges, one per rank, with no exchange on the data path. The one collective is an
all-gather of output shards, used to validate a sharded run against a single-device result.
One process per GPU; torch.distributed (NCCL on GPUs, gloo on CPU) is the plumbing.
"""

from __future__ import annotations


def split_rows(total: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous row range [begin, end) of `rank`; sizes differ by at most one row."""
    if world <= 0 or not 0 <= rank < world or total < 0:
        raise ValueError(f"bad split: total={total} world={world} rank={rank}")
    base, rem = divmod(total, world)
    begin = rank * base + min(rank, rem)
    return begin, begin + base + (1 if rank < rem else 0)


def all_gather_rows(shard, total: int, group=None):
    """Gathers every rank's row shard (split_rows layout) into the full [total, ...] tensor on
    every rank. Shards may differ by one row, so each is padded to the largest and trimmed."""
    import torch
    import torch.distributed as dist

    if shard.dtype in (torch.bfloat16, torch.float16, torch.int16):
        # gloo gathers neither 16-bit type: move the rows as bytes and view them back
        raw = shard.contiguous().view(torch.uint8)
        return all_gather_rows(raw, total, group).view(shard.dtype)
    world = dist.get_world_size(group)
    sizes = [split_rows(total, world, r) for r in range(world)]
    longest = max(e - b for b, e in sizes)
    padded = torch.zeros((longest, *shard.shape[1:]), dtype=shard.dtype, device=shard.device)
    padded[: shard.shape[0]] = shard
    parts = [torch.empty_like(padded) for _ in range(world)]
    dist.all_gather(parts, padded.contiguous(), group=group)
    return torch.cat([p[: e - b] for p, (b, e) in zip(parts, sizes)], dim=0)
