"""Self-play frames around the search step (scacchi/play.py:24-33, 93-175).

``play_training`` runs ``max_num_steps`` frames of a batch of games: each
frame asks the player (search + action commitment) for an action and the
posterior targets, steps every game, and resets the finished ones with a
fresh initial position while the frame keeps the finishing transition's
terminal flag and reward (pgx.experimental.auto_reset).  All state stays
on the device; the loop is plain Python over kernel launches.
"""

from __future__ import annotations

from typing import Any, NamedTuple

import numpy as np
import torch

from . import random as srandom
from .play_search import PosteriorTargets


class TrainingSamples(NamedTuple):
    """play.py:24-33, batch-major [B, T, ...]."""

    obs: torch.Tensor
    reward: torch.Tensor
    terminated: torch.Tensor
    discount: torch.Tensor
    posterior: PosteriorTargets
    played_action: torch.Tensor
    legal_action_mask: torch.Tensor
    psk_terminated: torch.Tensor | None = None


def _where(mask: torch.Tensor, a, b):
    """Row-wise select between two batched states of the same structure."""
    def pick(x, y):
        m = mask.reshape(mask.shape + (1,) * (x.dim() - 1))
        return torch.where(m, x, y)

    return type(a)(*[pick(x, y) for x, y in zip(a, b)])


def auto_reset_step(env, state, action: torch.Tensor, keys: np.ndarray):
    """pgx.experimental.auto_reset(env.step, env.init) for a batch: per lane
    key -> (step key, init key); a finished game restarts from env.init of
    its init key, keeping the finishing terminal flag and rewards."""
    zero_rewards = torch.zeros_like(state.rewards)
    done = state.terminated
    state = state._replace(terminated=torch.zeros_like(done), rewards=torch.where(done[:, None], zero_rewards,
                                                                                    state.rewards))
    stepped = env.step(state, action)
    finished = torch.nonzero(stepped.terminated).flatten().cpu().numpy()
    if finished.size == 0:
        return stepped
    init_keys = np.zeros((len(keys), 2), np.uint32)
    for i in finished:  # only the finished lanes' init keys are used
        init_keys[i] = srandom.split(keys[i])[1]
    fresh = env.init(init_keys)
    fresh = fresh._replace(terminated=stepped.terminated, rewards=stepped.rewards)
    return _where(stepped.terminated, fresh, stepped)


def selfplay_step_frame(env: Any, player, env_state, key) -> tuple[Any, dict]:
    """play.py:93-138: one frame of self-play."""
    player_key, reset_key = srandom.split(key)
    B = env_state.terminated.shape[0]
    # a reset state still carries the previous transition's terminal flag and
    # rewards for one frame; the player analyses the fresh board without them
    env_state = env_state._replace(terminated=torch.zeros_like(env_state.terminated),
                                   rewards=torch.zeros_like(env_state.rewards))
    observation = env_state.observation
    legal_action_mask = env_state.legal_action_mask
    output = player(env_state, player_key)
    if output.posterior is None:
        raise ValueError("self-play player must return posterior targets")
    actor = env_state.current_player.long()
    reset_keys = srandom.split(reset_key, B)
    env_state = auto_reset_step(env, env_state, output.action, reset_keys)
    reward = env_state.rewards[torch.arange(B, device=actor.device), actor]
    discount = torch.where(env_state.terminated, torch.zeros_like(reward), -torch.ones_like(reward))
    frame = dict(obs=observation, reward=reward, terminated=env_state.terminated, legal_action_mask=legal_action_mask,
                 discount=discount, posterior=output.posterior, played_action=output.action,
                 psk_terminated=torch.zeros_like(env_state.terminated))
    return env_state, frame


def _stack(frames: list, key: str):
    first = frames[0][key]
    if isinstance(first, torch.Tensor):
        return torch.stack([f[key] for f in frames], dim=1)
    return first


def _stack_tree(values: list):
    first = values[0]
    if first is None:
        return None
    if isinstance(first, torch.Tensor):
        return torch.stack(values, dim=1)
    return type(first)(*[_stack_tree([v[i] for v in values]) for i in range(len(first))])


def play_training(env: Any, player, rng_key, *, batch_size: int, max_num_steps: int) -> TrainingSamples:
    """play.py:141-175: ``max_num_steps`` frames of ``batch_size`` games."""
    rollout_rng, init_key = srandom.split(rng_key)
    env_state = env.init(srandom.split(init_key, batch_size))
    step_keys = srandom.split(rollout_rng, max_num_steps)
    frames = []
    for t in range(max_num_steps):
        env_state, frame = selfplay_step_frame(env, player, env_state, step_keys[t])
        frames.append(frame)
    return TrainingSamples(
        obs=_stack(frames, "obs"), reward=_stack(frames, "reward"), terminated=_stack(frames, "terminated"),
        discount=_stack(frames, "discount"), posterior=_stack_tree([f["posterior"] for f in frames]),
        played_action=_stack(frames, "played_action"), legal_action_mask=_stack(frames, "legal_action_mask"),
        psk_terminated=_stack(frames, "psk_terminated"))
