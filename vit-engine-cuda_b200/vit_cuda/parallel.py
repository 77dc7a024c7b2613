"""Batch data parallelism across the GPUs of one node.

ViT-B/16 inference shards by image: every rank holds a full replica of the
weights (346 MB fp32 + 692 MB of TF32 pairs), runs its contiguous slice of the
batch through the fused forward, and one NCCL all-gather assembles the logits
on every rank. There is no other exchange: images are independent and no
reduction crosses ranks. From 7 images per rank (224²) every kernel's
per-image arithmetic is the one a single GPU uses for the whole batch (CTA-pair
GEMM tiles, the two-tile attention, the fused head), so the gathered logits
equal the single-GPU ones bit for bit; smaller shards take the small-batch
kernels (split K, one query tile per CTA) and agree to FP32 rounding.
The reference project has no multi-GPU code; this module is new.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def shard_bounds(total: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous [start, end) rows of `total` for `rank`; the first
    total % world ranks take one extra row."""
    if world <= 0 or not 0 <= rank < world or total < 0:
        raise ValueError("shard_bounds: bad world/rank/total")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def padded_rows(total: int, world: int) -> int:
    """Rows per rank in the all-gather buffer (all ranks send the same size)."""
    return -(-total // world) if world > 0 else 0


def gather_rows(local: torch.Tensor, total: int, group=None) -> torch.Tensor:
    """All-gathers each rank's [rows_r, C] slice into [total, C] on every rank.

    Slices are padded to a common row count for all_gather_into_tensor and the
    padding is dropped afterwards, so uneven shards work."""
    if not dist.is_available() or not dist.is_initialized():
        return local
    world = dist.get_world_size(group)
    if world == 1:
        return local
    rank = dist.get_rank(group)
    per = padded_rows(total, world)
    start, end = shard_bounds(total, world, rank)
    if local.shape[0] != end - start:
        raise RuntimeError(
            f"gather_rows: rank {rank} holds {local.shape[0]} rows, expected {end - start}")
    send = torch.zeros((per,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    send[: local.shape[0]] = local
    recv = torch.empty((per * world,) + tuple(local.shape[1:]), dtype=local.dtype,
                       device=local.device)
    dist.all_gather_into_tensor(recv, send, group=group)
    pieces = []
    for r in range(world):
        s, e = shard_bounds(total, world, r)
        pieces.append(recv[r * per: r * per + (e - s)])
    return torch.cat(pieces, dim=0)


class DataParallelViT:
    """Runs `model` (a ViTCUDA, or any callable images -> [rows, C]) on this
    rank's slice of a global batch and all-gathers the logits."""

    def __init__(self, model, group=None):
        self.model = model
        self.group = group

    def local_slice(self, total: int) -> tuple[int, int]:
        if not dist.is_available() or not dist.is_initialized():
            return 0, total
        return shard_bounds(total, dist.get_world_size(self.group), dist.get_rank(self.group))

    def __call__(self, images: torch.Tensor) -> torch.Tensor:
        total = images.shape[0]
        start, end = self.local_slice(total)
        local = self.model(images[start:end])
        return gather_rows(local, total, self.group)
