"""Data-parallel plumbing: one process per GPU, the global batch split contiguously by image index.

The reference trains one image at a time over the whole batch (YoloTrainer.Train,
src/SimdYolo.Training/YoloTrainer.cs:185-199), and each image's BatchNorm statistics and loss
normalisation are its own (HeadOperations.cs:153-193, DetectionLoss.cs:92-98), so images are
independent units: rank r steps images [r * B, (r + 1) * B) of a global batch of world * B images.
The only exchange is inside the session (NCCL all-reduce of the gradient bucket and the step's
scalars, all-gather of the per-image BatchNorm statistics).  This module is the host side around
it: the NCCL id broadcast over the caller's control-plane process group, the shard arithmetic and
the max-over-ranks reduction of timings.
"""
from __future__ import annotations

from typing import Callable, Sequence, Tuple

import numpy as np


def shard_range(global_batch: int, rank: int, world: int) -> Tuple[int, int]:
    """[start, stop) of rank's images.  Every rank steps the same number of images (the session
    folds BatchNorm running statistics rank by rank, `images` per rank)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} / world {world}")
    if global_batch % world:
        raise ValueError(f"global batch {global_batch} is not a multiple of {world} ranks")
    per = global_batch // world
    return rank * per, (rank + 1) * per


def shard(images: np.ndarray, boxes_per_image: Sequence, rank: int, world: int):
    """This rank's slice of a global batch: (images[start:stop], boxes_per_image[start:stop])."""
    if len(images) != len(boxes_per_image):
        raise ValueError("images and box lists differ in length")
    a, b = shard_range(len(images), rank, world)
    return images[a:b], list(boxes_per_image[a:b])


def broadcast_nccl_id(dist, rank: int, make_id: Callable[[], bytes] | None = None) -> bytes:
    """Rank 0 makes the NCCL unique id, every rank of the control-plane group receives it."""
    if make_id is None:
        from . import nccl_unique_id as make_id
    obj = [make_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    nid = obj[0]
    if not isinstance(nid, (bytes, bytearray)) or len(nid) != 128:
        raise RuntimeError("NCCL unique id must be 128 bytes")
    return bytes(nid)


def create_session(dist, model: str, local_rank: int, per_rank_batch: int, **config):
    """A Session for this rank of the control-plane group `dist` (None or world 1: single GPU)."""
    from . import Session, make_config

    world = dist.get_world_size() if dist is not None and dist.is_initialized() else 1
    rank = dist.get_rank() if world > 1 else 0
    nid = broadcast_nccl_id(dist, rank) if world > 1 else b""
    cfg = make_config(model, max_batch=per_rank_batch, device=local_rank, rank=rank, world_size=world, nccl_id=nid,
                      **config)
    return Session(cfg)


def max_over_ranks(dist, value: float) -> float:
    """Largest value over the ranks of the control-plane group (a device time is the slowest rank's)."""
    if dist is None or not dist.is_initialized() or dist.get_world_size() == 1:
        return float(value)
    import torch

    t = torch.tensor([float(value)], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
