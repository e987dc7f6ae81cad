"""Seeded synthetic game: the isolated search-kernel workload.

Hex 9x9 action space (82 actions = 81 cells + swap); network outputs are
synthesised from the state (csrc/synthetic_env.h): prior logits N(0, 1),
value/Q log-concentrations clip(N(0.5, 1), -4, 6) per outcome with
alpha = exp(.), legal masks Bernoulli(0.7) with at least one legal move, and
about 1 % of lanes near-degenerate (every alpha = 1e-3).  A small terminal
probability can be switched on to exercise certificate propagation.

``SyntheticGame`` is both a recurrent function (callable with the reference's
signature) and a native one: ``native_search`` runs the whole simulation loop
inside the CUDA library.
"""

from __future__ import annotations

import ctypes as C
import dataclasses
from typing import NamedTuple

import numpy as np
import torch

from . import _lib
from . import random as srandom
from .dirichlet_mctx.base import RecurrentFnOutput, RootFnOutput
from .dirichlet_mctx.tree import Tree, ptr, stream_handle

STATE_BYTES = 16


@dataclasses.dataclass(frozen=True)
class SyntheticGameConfig:
    seed: int = 0
    num_actions: int = 82
    legal_prob: float = 0.7
    terminal_prob: float = 0.0
    degenerate_lane_prob: float = 0.01
    degenerate_alpha: float = 1e-3
    logc_mean: float = 0.5
    logc_std: float = 1.0
    logc_min: float = -4.0
    logc_max: float = 6.0

    def params(self) -> _lib.SyntheticParams:
        k = srandom.PRNGKey(self.seed)
        return _lib.SyntheticParams(int(k[0]), int(k[1]), self.num_actions, self.legal_prob, self.terminal_prob,
                                    self.degenerate_lane_prob, self.degenerate_alpha, self.logc_mean,
                                    self.logc_std, self.logc_min, self.logc_max)


class SyntheticState(NamedTuple):
    """pgx.State-shaped root state of the synthetic game (the fields the
    search boundary reads).  ``observation`` is the 16-byte state record."""

    observation: torch.Tensor
    legal_action_mask: torch.Tensor
    current_player: torch.Tensor
    rewards: torch.Tensor
    terminated: torch.Tensor


class SyntheticGame:
    def __init__(self, config: SyntheticGameConfig = SyntheticGameConfig(), device="cuda"):
        self.config = config
        self.device = torch.device(device)
        self._params = config.params()
        self._ws = None

    @property
    def num_actions(self) -> int:
        return self.config.num_actions

    def root(self, batch: int) -> RootFnOutput:
        """Root network outputs and states for `batch` lanes."""
        A, dev = self.num_actions, self.device
        logits = torch.empty((batch, A), dtype=torch.float32, device=dev)
        value = torch.empty((batch, 2), dtype=torch.float32, device=dev)
        av = torch.empty((batch, A, 2), dtype=torch.float32, device=dev)
        inv = torch.empty((batch, A), dtype=torch.uint8, device=dev)
        term = torch.empty((batch,), dtype=torch.int8, device=dev)
        tp = torch.empty((batch,), dtype=torch.int32, device=dev)
        emb = torch.empty((batch, STATE_BYTES), dtype=torch.uint8, device=dev)
        _lib.check(_lib.lib().scacchi_synthetic_root(C.byref(self._params), batch, ptr(logits), ptr(value), ptr(av),
                                                     ptr(inv), ptr(term), ptr(tp), ptr(emb), stream_handle(dev)),
                   "synthetic_root")
        logits = torch.where(inv.bool(), torch.full_like(logits, -float("inf")), logits)
        return RootFnOutput(prior_logits=logits, value=value, action_values=av, embedding=emb,
                            terminal_outcome=term, to_play=tp)

    def __call__(self, params, rng_key, action: torch.Tensor, embedding: torch.Tensor):
        """recurrent_fn(params, key, action, parent_state) -> (step, child_state)."""
        B, A, dev = action.shape[0], self.num_actions, self.device
        value = torch.empty((B, 2), dtype=torch.float32, device=dev)
        av = torch.empty((B, A, 2), dtype=torch.float32, device=dev)
        inv = torch.empty((B, A), dtype=torch.uint8, device=dev)
        term = torch.empty((B,), dtype=torch.int8, device=dev)
        tp = torch.empty((B,), dtype=torch.int32, device=dev)
        child = torch.empty((B, STATE_BYTES), dtype=torch.uint8, device=dev)
        act = action.to(device=dev, dtype=torch.int32).contiguous()
        emb = embedding.to(device=dev, dtype=torch.uint8).contiguous()
        _lib.check(_lib.lib().scacchi_synthetic_recurrent(C.byref(self._params), B, ptr(act), ptr(emb), ptr(value),
                                                          ptr(av), ptr(inv), ptr(term), ptr(tp), ptr(child),
                                                          stream_handle(dev)), "synthetic_recurrent")
        return RecurrentFnOutput(value=value, action_values=av, invalid_actions=inv.bool(), terminal_outcome=term,
                                 to_play=tp), child

    def native_search(self, tree: Tree, keys: torch.Tensor, num_simulations: int, max_depth: int,
                      params: _lib.UpdateParams, stats: torch.Tensor | None) -> None:
        if tree.E != STATE_BYTES or tree.A != self.num_actions:
            raise ValueError("tree was not built from this game's root")
        need = int(_lib.lib().scacchi_search_workspace_bytes(tree.batch, tree.A, tree.E))
        if self._ws is None or self._ws.numel() < need or self._ws.device != tree.device:
            self._ws = torch.empty((need,), dtype=torch.uint8, device=tree.device)
        _lib.check(_lib.lib().scacchi_search_synthetic(
            tree.sref(), C.byref(self._params), ptr(keys), int(num_simulations), int(max_depth), C.byref(params),
            ptr(self._ws), ptr(stats), stream_handle(tree.device)), "search_synthetic")

    def init(self, batch: int) -> SyntheticState:
        """Root states of `batch` lanes (lane b is state b of the seeded game)."""
        root = self.root(batch)
        dev = self.device
        return SyntheticState(observation=root.embedding, legal_action_mask=torch.isfinite(root.prior_logits),
                              current_player=root.to_play, rewards=torch.zeros((batch, 2), device=dev),
                              terminated=torch.zeros((batch,), dtype=torch.bool, device=dev))

    def evaluator(self, observation: torch.Tensor):
        """The synthetic network on state records [B, 16] -> EvaluatorOutput."""
        from .play_search import EvaluatorOutput

        B, A, dev = observation.shape[0], self.num_actions, self.device
        logits = torch.empty((B, A), dtype=torch.float32, device=dev)
        value = torch.empty((B, 2), dtype=torch.float32, device=dev)
        av = torch.empty((B, A, 2), dtype=torch.float32, device=dev)
        inv = torch.empty((B, A), dtype=torch.uint8, device=dev)
        term = torch.empty((B,), dtype=torch.int8, device=dev)
        tp = torch.empty((B,), dtype=torch.int32, device=dev)
        obs = observation.to(device=dev, dtype=torch.uint8).contiguous()
        _lib.check(_lib.lib().scacchi_synthetic_evaluate(C.byref(self._params), B, ptr(obs), ptr(logits),
                                                         ptr(value), ptr(av), ptr(inv), ptr(term), ptr(tp),
                                                         stream_handle(dev)), "synthetic_evaluate")
        logits = torch.where(inv.bool(), torch.full_like(logits, -float("inf")), logits)
        mean = value / value.sum(-1, keepdim=True)
        return EvaluatorOutput(logits=logits, value=mean[:, 1] - mean[:, 0], alpha_v=value, alpha_q=av)

    def native_recurrent_fn(self, evaluator) -> "SyntheticGame":
        """The game's own fused step + evaluation (runs natively)."""
        return self

    def embedding(self, state: SyntheticState) -> torch.Tensor:
        return state.observation
