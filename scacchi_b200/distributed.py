"""Lane sharding of the search step over the GPUs of one node.

Lanes are independent games, so every rank searches its own local batch
with no communication inside the step (the reference runs one local batch
per device under a shard map: play.py:219-244, distributed.py:62-97).  The
only collective is the gather of the root targets at the end of the step.

One process per GPU; the process group is ``torch.distributed`` (NCCL on
GPUs, gloo for the CPU tests).
"""

from __future__ import annotations

import dataclasses
import os

import torch
import torch.distributed as dist

from . import random as R
from .play_search import PosteriorPrediction, PosteriorTargets, TargetMetadata


@dataclasses.dataclass(frozen=True)
class LaneSharding:
    """Rank ``rank`` of ``world`` owns lanes [rank * L, (rank + 1) * L)."""

    world: int = 1
    rank: int = 0

    @classmethod
    def from_env(cls) -> "LaneSharding":
        return cls(int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")))

    def local_batch_size(self, batch_size: int) -> int:
        """distributed.py:62-70: the global batch must split evenly."""
        if batch_size % self.world != 0:
            raise ValueError("batch size must be divisible by the batch-parallel device "
                             f"count ({self.world}).")
        return batch_size // self.world

    def lane_range(self, batch_size: int) -> tuple[int, int]:
        local = self.local_batch_size(batch_size)
        return self.rank * local, (self.rank + 1) * local

    def device_key(self, rng_key):
        """play.py:231,243: the per-device key is split(rng_key, D)[d]."""
        return R.split(rng_key, self.world)[self.rank]


def _gather(t: torch.Tensor, world: int, group=None) -> torch.Tensor:
    t = t.contiguous()
    if dist.get_backend(group) == "nccl":
        out = torch.empty((world * t.shape[0],) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
        dist.all_gather_into_tensor(out, t, group=group)
        return out
    parts = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(parts, t, group=group)
    return torch.cat(parts)


PREDICTION_FIELDS = ("policy", "alpha_v", "alpha_q")
METADATA_FIELDS = ("search_action", "q_target_kind", "q_target_weight", "q_target_outcome", "q_target_distance",
                   "v_target_kind", "v_target_weight", "v_target_outcome", "v_target_distance")


def gather_targets(targets: PosteriorTargets, sharding: LaneSharding, group=None) -> PosteriorTargets:
    """All-gather the root targets of every rank in rank (= lane) order.

    Every rank issues the same collectives in the same order: the fields
    gathered are the ones present, and presence is decided by the search
    configuration, which all ranks share.  A world of one returns the
    targets unchanged."""
    if sharding.world == 1:
        return targets
    pred = targets.prediction
    new_pred = pred._replace(**{f: _gather(getattr(pred, f), sharding.world, group)
                                for f in PREDICTION_FIELDS if getattr(pred, f) is not None})
    meta = targets.metadata
    if meta is not None:
        meta = meta._replace(**{f: _gather(getattr(meta, f), sharding.world, group)
                                for f in METADATA_FIELDS if getattr(meta, f) is not None})
    return PosteriorTargets(prediction=new_pred, metadata=meta)


__all__ = ["LaneSharding", "gather_targets", "PosteriorPrediction", "PosteriorTargets", "TargetMetadata"]
