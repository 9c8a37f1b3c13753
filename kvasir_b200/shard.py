"""Independent-sequence sharding across ranks (one process per GPU).

Sequences are split into contiguous, as-equal-as-possible blocks; each rank
keeps a full weight replica and the KV cache of its block, and no data moves
between ranks during a step.  The only exchange is the gather of sampled token
ids, done on the host after the steps (`gather_ids`), over whatever
torch.distributed backend the process group uses (gloo on CPU tests).
"""
from __future__ import annotations

import torch


def shard_sequences(n_total: int, world: int, rank: int) -> tuple[int, int]:
    """(first sequence, count) owned by `rank`."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    base, extra = divmod(n_total, world)
    start = rank * base + min(rank, extra)
    return start, base + (1 if rank < extra else 0)


def gather_ids(local_ids: torch.Tensor, n_total: int, group=None) -> torch.Tensor:
    """All ranks' [steps, local] int32 id blocks -> [steps, n_total] in
    sequence order (every rank receives the full table)."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    steps = local_ids.shape[0]
    width = -(-n_total // world)  # ceil: pad every block to the same width
    pad = torch.full((steps, width), -1, dtype=torch.int32)
    pad[:, :local_ids.shape[1]] = local_ids
    parts = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(parts, pad, group=group)
    out = torch.empty((steps, n_total), dtype=torch.int32)
    for r, p in enumerate(parts):
        s, c = shard_sequences(n_total, world, r)
        out[:, s:s + c] = p[:, :c]
    return out
