"""simulate -> expand -> backward on the device tree (search.py of the reference).

The loop over simulations runs on the host and issues one kernel per phase
(simulate, expand, backward) plus the recurrent function.  Recurrent
functions that implement ``native_search`` (the built-in games) run the whole
loop inside the C library instead, with no Python in between.
"""

from __future__ import annotations

import ctypes as C
from typing import Any, Callable

import numpy as np
import torch

from .. import _lib
from .. import random as srandom
from .base import RecurrentFnOutput, RootFnOutput
from .posterior_updates import rule_params, update_posterior
from .tree import Tree, _init_tree, ptr, stream_handle


class PhaseTimer:
    """CUDA events around the phases of the host-driven loop (simulate,
    recurrent, expand, backward), recorded on the current stream; install
    with ``set_phase_timer``.  Measurement only: the loop records nothing
    when no timer is installed."""

    PHASES = ("simulate", "recurrent", "expand", "backward")

    def __init__(self):
        self.marks = []

    def mark(self) -> None:
        e = torch.cuda.Event(enable_timing=True)
        e.record(torch.cuda.current_stream())
        self.marks.append(e)

    def totals_ms(self) -> dict:
        """Summed milliseconds per phase over every simulation timed so far."""
        torch.cuda.synchronize()
        out = {p: 0.0 for p in self.PHASES}
        for i in range(0, len(self.marks) - 4, 5):
            for j, p in enumerate(self.PHASES):
                out[p] += self.marks[i + j].elapsed_time(self.marks[i + j + 1])
        return out

    def reset(self) -> None:
        self.marks = []


_PHASE_TIMER: PhaseTimer | None = None


def set_phase_timer(timer: PhaseTimer | None) -> None:
    global _PHASE_TIMER
    _PHASE_TIMER = timer


class SimulationBuffers:
    """Per-simulation device buffers: Simulation + recurrent outputs."""

    def __init__(self, B: int, A: int, E: int, device):
        i32, u8 = torch.int32, torch.uint8
        self.parent = torch.empty((B,), dtype=i32, device=device)
        self.action = torch.empty((B,), dtype=i32, device=device)
        self.active = torch.empty((B,), dtype=u8, device=device)
        self.parent_embedding = torch.empty((B, max(E, 1)), dtype=u8, device=device)


def _c(t, dtype, device):
    return torch.as_tensor(t).to(device=device, dtype=dtype).contiguous()


def simulate(tree: Tree, simulate_key: torch.Tensor, max_depth: int, bufs: SimulationBuffers,
             stats: torch.Tensor | None = None) -> None:
    """search.py:21-78 for every lane; ``simulate_key`` is a device uint32[2].
    ``stats``: optional device int64[2] (nodes selected from, child priors
    gathered)."""
    _lib.check(_lib.lib().scacchi_simulate(
        tree.sref(), ptr(simulate_key), int(max_depth), ptr(bufs.parent), ptr(bufs.action), ptr(bufs.active),
        ptr(bufs.parent_embedding) if tree.E else None, ptr(stats), stream_handle(tree.device)), "simulate")


def expand(tree: Tree, new_node: int, bufs: SimulationBuffers, step: RecurrentFnOutput,
           child_embedding: torch.Tensor | None, lazy_init: bool = True):
    """search.py:101-143 with the recurrent outputs already computed."""
    dev = tree.device
    B, A = tree.batch, tree.A
    v = _c(step.value, torch.float32, dev)
    av = _c(step.action_values, torch.float32, dev)
    if tuple(v.shape) != (B, 2) or tuple(av.shape) != (B, A, 2):
        raise ValueError(f"recurrent_fn returned value {tuple(v.shape)} / action_values {tuple(av.shape)}; "
                         f"expected ({B}, 2) / ({B}, {A}, 2)")
    inv = _c(step.invalid_actions, torch.uint8, dev)
    term = _c(step.terminal_outcome, torch.int8, dev)
    tp = _c(step.to_play, torch.int32, dev)
    _lib.check(_lib.lib().scacchi_expand(
        tree.sref(), int(new_node), ptr(bufs.parent), ptr(bufs.action), ptr(bufs.active), ptr(v), ptr(av),
        ptr(inv), ptr(term), ptr(tp), ptr(child_embedding), int(lazy_init), stream_handle(dev)), "expand")
    return v, tp


def backward(tree: Tree, backward_key: torch.Tensor, bufs: SimulationBuffers, step_value: torch.Tensor,
             step_to_play: torch.Tensor, params: _lib.UpdateParams, stats: torch.Tensor | None = None):
    """search.py:146-171 with the rule of ``params``.  ``stats``: optional
    device int64[3] (node updates, visited children gathered, Monte Carlo
    fallbacks)."""
    _lib.check(_lib.lib().scacchi_backward(
        tree.sref(), ptr(backward_key), ptr(bufs.parent), ptr(bufs.action), ptr(bufs.active), ptr(step_value),
        ptr(step_to_play), C.byref(params), ptr(stats), stream_handle(tree.device)), "backward")


def validate(num_simulations: int, max_depth: int | None) -> int:
    """search.py:192-198."""
    if num_simulations < 0:
        raise ValueError(f"num_simulations must be >= 0, got {num_simulations}")
    if max_depth is None:
        max_depth = num_simulations
    if num_simulations > 0 and max_depth < 1:
        raise ValueError(f"max_depth must be >= 1 when num_simulations is positive, got {max_depth}")
    return max(1, int(max_depth))


def search(params: Any, rng_key, *, root: RootFnOutput, recurrent_fn: Callable,
           posterior_update: Callable = update_posterior, num_simulations: int, max_depth: int | None = None,
           invalid_actions: torch.Tensor | None = None, stats: torch.Tensor | None = None,
           action_selection_fn: Callable | None = None, loop_fn: Callable | None = None) -> Tree:
    """search.py:189-251.  ``action_selection_fn`` and ``loop_fn`` exist in the
    reference's signature; only the built-in Thompson selector and a plain
    loop are supported.  ``stats``: optional device int64[6] work counters
    (backward [0..2], simulate [4..5])."""
    if action_selection_fn is not None and getattr(action_selection_fn, "__name__", "") != \
            "thompson_action_selection":
        raise ValueError("the native search uses the built-in Thompson action selection only")
    max_depth = validate(num_simulations, max_depth)
    rparams = rule_params(posterior_update)
    if invalid_actions is None:
        invalid_actions = ~torch.isfinite(root.prior_logits)
    tree = _init_tree(root, num_simulations, invalid_actions, full=False)
    if num_simulations == 0:
        return tree
    dev = tree.device
    sched = srandom.key_schedule(rng_key, num_simulations)
    keys = torch.from_numpy(sched.view(np.int32)).to(dev, non_blocking=False)
    if hasattr(recurrent_fn, "native_search"):
        recurrent_fn.native_search(tree, keys, num_simulations, max_depth, rparams, stats)
        return tree
    bufs = SimulationBuffers(tree.batch, tree.A, tree.E, dev)
    timer = _PHASE_TIMER
    for i in range(num_simulations):
        if timer is not None:
            timer.mark()
        simulate(tree, keys[i, 1], max_depth, bufs, None if stats is None else stats[4:])
        if timer is not None:
            timer.mark()
        embedding = tree.codec.unpack(bufs.parent_embedding[:, :tree.E]) if tree.codec is not None else None
        step, child = recurrent_fn(params, sched[i, 2], bufs.action, embedding)
        child_bytes = None
        if tree.codec is not None and tree.E:
            child_bytes = tree.codec.pack(child, tree.batch, dev)
        if timer is not None:
            timer.mark()
        v, tp = expand(tree, i + 1, bufs, step, child_bytes)
        if timer is not None:
            timer.mark()
        backward(tree, keys[i, 3], bufs, v, tp, rparams, stats)
        if timer is not None:
            timer.mark()
    return tree
