"""Data-parallel plumbing for the SC ViT forward across the GPUs of one box.

The reference runs one independent process per GPU over contiguous data
shards and merges the per-shard predictions offline
(``det/run_coco_val_8gpu.sh:1-60``, ``det/merge_shards.py:1-80``).  Here the
same partition is one ``torch.distributed`` job: rank r takes the r-th
contiguous slice of the image batch, weights and SC pools are replicated
(identical by seed on every rank), and the only collective is a gather of
the fp32 logits (NCCL over NVLink; gloo on CPU for tests).
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist

__all__ = ["shard_range", "gather_logits"]


def shard_range(global_batch: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous [start, stop) of the images rank ``rank`` processes; the
    first ``global_batch % world`` ranks take one extra image."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    base, extra = divmod(int(global_batch), world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def gather_logits(local: torch.Tensor, global_batch: int, world: int,
                  out: Optional[torch.Tensor] = None, group=None) -> torch.Tensor:
    """All ranks' logits in rank order, ``[global_batch, C]`` on every rank.

    Equal shards use one ``all_gather_into_tensor`` (the NCCL fast path);
    ragged shards pad to the largest shard and trim."""
    if world == 1:
        if out is not None:
            out.copy_(local)
            return out
        return local
    C = local.shape[-1]
    sizes = [shard_range(global_batch, r, world) for r in range(world)]
    counts = [b - a for a, b in sizes]
    if len(set(counts)) == 1 and dist.get_backend(group) == "nccl":
        if out is None:
            out = torch.empty(global_batch, C, dtype=local.dtype, device=local.device)
        dist.all_gather_into_tensor(out, local.contiguous(), group=group)
        return out
    top = max(counts)
    pad = torch.zeros(top, C, dtype=local.dtype, device=local.device)
    pad[: local.shape[0]] = local
    parts = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(parts, pad, group=group)
    res = torch.cat([p[:c] for p, c in zip(parts, counts)], dim=0)
    if out is not None:
        out.copy_(res)
        return out
    return res
