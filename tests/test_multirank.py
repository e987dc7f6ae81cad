"""The N > 1 lane-sharded path on CPU: two gloo ranks, the oracle as the
per-rank search, the same key split and target gather that bench.py uses
on NCCL."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import oracle as O
from scacchi_b200 import random as R
from scacchi_b200.distributed import LaneSharding, gather_targets
from scacchi_b200.play_search import PosteriorPrediction, PosteriorTargets, TargetMetadata

GLOBAL_LANES, SIMS, WORLD = 12, 6, 2


def _local_targets(sharding: LaneSharding) -> PosteriorTargets:
    """One rank's search on its own local batch (game seed = rank, as in
    bench.py), packed as root targets on CPU tensors."""
    local = sharding.local_batch_size(GLOBAL_LANES)
    env = O.synth_params(seed=sharding.rank, terminal_prob=0.05)
    out = O.search_synthetic(env, local, sharding.device_key(O.PRNGKey(0)), SIMS,
                             O.Rule(prefix_cdf=True, kappa=1.0, samples=8), max_depth=SIMS, policy_samples=8)
    s = out.search_tree.summary()
    return PosteriorTargets(
        prediction=PosteriorPrediction(policy=torch.from_numpy(out.action_weights),
                                       alpha_v=torch.from_numpy(s["value_alpha"]),
                                       alpha_q=torch.from_numpy(s["alpha"])),
        metadata=TargetMetadata(search_action=torch.from_numpy(out.action),
                                q_target_outcome=torch.from_numpy(s["q_categorical_outcome"]),
                                q_target_distance=torch.from_numpy(s["q_categorical_distance"]),
                                v_target_outcome=torch.from_numpy(s["v_categorical_outcome"]),
                                v_target_distance=torch.from_numpy(s["v_categorical_distance"])))


def _rank_main(rank, port, result_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        sharding = LaneSharding(WORLD, rank)
        g = gather_targets(_local_targets(sharding), sharding)
        if rank == 0:
            arrays = {f"prediction.{k}": v.numpy() for k, v in g.prediction._asdict().items() if v is not None}
            arrays.update({f"metadata.{k}": v.numpy() for k, v in g.metadata._asdict().items() if v is not None})
            np.savez(result_path, **arrays)
    finally:
        dist.destroy_process_group()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_rank_gather_equals_sequential_shards(tmp_path):
    path = str(tmp_path / "gathered.npz")
    mp.start_processes(_rank_main, args=(_free_port(), path), nprocs=WORLD, join=True, start_method="spawn")
    got = np.load(path)
    shards = [_local_targets(LaneSharding(WORLD, r)) for r in range(WORLD)]
    for name in got.files:
        part, field = name.split(".")
        want = np.concatenate([getattr(getattr(t, part), field).numpy() for t in shards])
        assert np.array_equal(got[name], want), name
    assert got["prediction.policy"].shape == (GLOBAL_LANES, 82)


def test_device_keys_and_lane_ranges():
    key = R.PRNGKey(0)
    keys = [LaneSharding(4, r).device_key(key) for r in range(4)]
    assert np.array_equal(np.stack([np.asarray(k) for k in keys]), np.asarray(R.split(key, 4)))
    assert [LaneSharding(4, r).lane_range(32) for r in range(4)] == [(0, 8), (8, 16), (16, 24), (24, 32)]
    with pytest.raises(ValueError, match="divisible"):
        LaneSharding(3, 0).local_batch_size(32)
    assert gather_targets("unchanged", LaneSharding(1, 0)) == "unchanged"
