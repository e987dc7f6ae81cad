"""Hex on the GPU, the environment of the full search step.

The reference's environment is pgx 2.6.0's Hex wrapped in
``scacchi/envs.py:98-125`` (random player order at init, swap always
masked).  ``HexGame`` offers the pgx-shaped fields the search boundary
reads (``observation``, ``legal_action_mask``, ``current_player``,
``rewards``, ``terminated``) and keeps the game itself in a 48-byte record
per lane (two bitboards plus turn state), which is also what the search
tree stores per node.  Its recurrent function runs the step, the
observation and the terminal-outcome derivation of
``dirichlet_q_search.py:43-76`` in one kernel, then calls the evaluator on
the child observations.
"""

from __future__ import annotations

import ctypes as C
from typing import Callable, NamedTuple

import numpy as np
import torch

from . import _lib
from . import random as srandom
from .dirichlet_mctx.base import RecurrentFnOutput
from .dirichlet_mctx.tree import ptr, stream_handle

RECORD_BYTES = 48


class HexState(NamedTuple):
    """pgx.State-shaped batch of Hex states."""

    observation: torch.Tensor        # float32 [B, size, size, 4]
    legal_action_mask: torch.Tensor  # bool [B, size * size + 1]
    current_player: torch.Tensor     # int32 [B]
    rewards: torch.Tensor            # float32 [B, 2]
    terminated: torch.Tensor         # bool [B]
    record: torch.Tensor             # uint8 [B, 48]


class HexGame:
    def __init__(self, size: int = 9, device="cuda"):
        if not 2 <= size <= 11:
            raise ValueError(f"Hex size must be in [2, 11], got {size}")
        self.size = int(size)
        self.device = torch.device(device)

    @property
    def num_actions(self) -> int:
        return self.size * self.size + 1

    # ---- states ---------------------------------------------------------
    def _empty_records(self, batch: int) -> torch.Tensor:
        return torch.empty((batch, RECORD_BYTES), dtype=torch.uint8, device=self.device)

    def init(self, keys) -> HexState:
        """env.init per lane key (envs.py:103-112); keys uint32 [B, 2]."""
        k = torch.as_tensor(np.ascontiguousarray(np.asarray(keys, np.uint32)).view(np.int32)).to(self.device)
        B = k.shape[0]
        rec = self._empty_records(B)
        _lib.check(_lib.lib().scacchi_hex_init(B, self.size, ptr(k), ptr(rec), stream_handle(self.device)),
                   "hex_init")
        return self.observe(rec)

    def random_roots(self, batch: int, key, min_moves: int = 0, max_moves: int = 20) -> HexState:
        """Seeded roots: per lane a random player order and min_moves to
        max_moves uniform random legal moves from the empty board."""
        k0, k1 = (int(v) for v in np.asarray(key, np.uint32).reshape(2))
        rec = self._empty_records(batch)
        _lib.check(_lib.lib().scacchi_hex_random_roots(batch, self.size, k0, k1, int(min_moves), int(max_moves),
                                                       ptr(rec), stream_handle(self.device)), "hex_random_roots")
        return self.observe(rec)

    def observe(self, record: torch.Tensor) -> HexState:
        B, s, A, dev = record.shape[0], self.size, self.num_actions, self.device
        rec = record.to(device=dev, dtype=torch.uint8).contiguous()
        obs = torch.empty((B, s, s, 4), dtype=torch.float32, device=dev)
        inv = torch.empty((B, A), dtype=torch.uint8, device=dev)
        tp = torch.empty((B,), dtype=torch.int32, device=dev)
        rew = torch.empty((B, 2), dtype=torch.float32, device=dev)
        term = torch.empty((B,), dtype=torch.uint8, device=dev)
        _lib.check(_lib.lib().scacchi_hex_observe(B, ptr(rec), ptr(obs), ptr(inv), None, ptr(tp), ptr(rew),
                                                  ptr(term), stream_handle(dev)), "hex_observe")
        return HexState(observation=obs, legal_action_mask=inv == 0, current_player=tp, rewards=rew,
                        terminated=term.bool(), record=rec)

    def step(self, state: HexState, action: torch.Tensor) -> HexState:
        """env.step (envs.py:114-123) for a batch of legal actions."""
        B, s, A, dev = state.record.shape[0], self.size, self.num_actions, self.device
        act = action.to(device=dev, dtype=torch.int32).contiguous()
        nxt = self._empty_records(B)
        obs = torch.empty((B, s, s, 4), dtype=torch.float32, device=dev)
        inv = torch.empty((B, A), dtype=torch.uint8, device=dev)
        tp = torch.empty((B,), dtype=torch.int32, device=dev)
        rew = torch.empty((B, 2), dtype=torch.float32, device=dev)
        term = torch.empty((B,), dtype=torch.uint8, device=dev)
        _lib.check(_lib.lib().scacchi_hex_step(B, ptr(state.record.contiguous()), ptr(act), ptr(nxt), ptr(obs),
                                               ptr(inv), None, ptr(tp), ptr(rew), ptr(term), stream_handle(dev)),
                   "hex_step")
        return HexState(observation=obs, legal_action_mask=inv == 0, current_player=tp, rewards=rew,
                        terminated=term.bool(), record=nxt)

    # ---- search hooks -----------------------------------------------------
    def embedding(self, state: HexState) -> torch.Tensor:
        """What the tree stores per node: the 48-byte record."""
        return state.record

    def native_recurrent_fn(self, evaluator: Callable) -> Callable:
        """dirichlet_q_search.py:43-76 with the step, observation and
        terminal outcome fused into one kernel; the evaluator runs on the
        child observations."""
        game = self

        def recurrent_fn(params, rng_key, action: torch.Tensor, embedding: torch.Tensor):
            del params, rng_key
            B, s, A, dev = action.shape[0], game.size, game.num_actions, game.device
            rec = embedding.to(device=dev, dtype=torch.uint8).contiguous()
            act = action.to(device=dev, dtype=torch.int32).contiguous()
            nxt = game._empty_records(B)
            obs = torch.empty((B, s, s, 4), dtype=torch.float32, device=dev)
            inv = torch.empty((B, A), dtype=torch.uint8, device=dev)
            term = torch.empty((B,), dtype=torch.int8, device=dev)
            tp = torch.empty((B,), dtype=torch.int32, device=dev)
            _lib.check(_lib.lib().scacchi_hex_step(B, ptr(rec), ptr(act), ptr(nxt), ptr(obs), ptr(inv), ptr(term),
                                                   ptr(tp), None, None, stream_handle(dev)), "hex_step")
            prediction = evaluator(obs)
            if prediction.alpha_v is None or prediction.alpha_q is None:
                raise ValueError("evaluator output is missing alpha_v or alpha_q")
            step = RecurrentFnOutput(value=prediction.alpha_v, action_values=prediction.alpha_q,
                                     invalid_actions=inv.bool(), terminal_outcome=term, to_play=tp)
            return step, nxt

        return recurrent_fn


def hex_error() -> int:
    """Sticky Hex flags (bit 0: a record with an out-of-range size)."""
    v = C.c_uint32(0)
    _lib.check(_lib.lib().scacchi_hex_error(C.byref(v)), "hex_error")
    return int(v.value)


def lane_keys(key, batch: int) -> np.ndarray:
    """split(key, batch): per-lane init keys, as a vmapped env.init uses."""
    return np.asarray(srandom.split(key, batch), np.uint32)
