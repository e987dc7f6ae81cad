"""ctypes wrapper around the C oracle (``oracle/oracle.c``).

TEST INFRASTRUCTURE ONLY: the checker for the CUDA search kernels and the
timed CPU baseline.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` import it.

The C code restates the reference's ``scacchi/dirichlet_mctx`` algorithm lane
by lane (file:line citations are in ``oracle.c``); this module only converts
numpy arrays.  Outcomes are binary (Hex).
"""

from __future__ import annotations

import ctypes as C
import dataclasses
import functools
import os
import subprocess
from typing import Callable, NamedTuple

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")

NO_OUTCOME = -1


def build() -> str:
    """Compile ``liboracle.so`` with the committed Makefile (gcc only)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


@functools.lru_cache(maxsize=None)
def lib() -> C.CDLL:
    if not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(
        os.path.join(_HERE, "oracle.c")
    ):
        build()
    return C.CDLL(_LIB_PATH)


def _p(a: np.ndarray | None):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data_as(C.c_void_p)


class PrefixParams(C.Structure):
    _fields_ = [
        ("half_width", C.c_int),
        ("tail_scale", C.c_float),
        ("min_half_range", C.c_float),
        ("max_half_range", C.c_float),
    ]


class UpdateParams(C.Structure):
    _fields_ = [
        ("rule", C.c_int),
        ("kappa_ge_one", C.c_int),
        ("inv_kappa", C.c_float),
        ("kappa", C.c_float),
        ("samples", C.c_int),
        ("prefix", PrefixParams),
        ("density_tol", C.c_float),
    ]


class PrefixOut(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in (
        "policy", "raw_policy", "raw_mass", "normalization_error", "finite",
        "grid_half_range", "tail_range_clipped", "density_log_integral",
        "fallback_interval_count")]


class TreeStruct(C.Structure):
    _fields_ = [("B", C.c_int), ("C", C.c_int), ("A", C.c_int), ("emb_bytes", C.c_int)] + [
        (n, C.c_void_p) for n in (
            "parents", "children", "to_play", "node_outcome", "node_payload",
            "edge_outcome", "edge_payload", "value_prior", "value_alpha",
            "edge_alpha", "invalid", "embedding")
    ] + [("lane_offset", C.c_int), ("total_batch", C.c_int)]


class ContextSoA(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in (
        "active", "leaf_active", "leaf_action", "leaf_value", "leaf_to_play",
        "node_to_play", "node_payload", "value_prior", "value_alpha", "edge_alpha",
        "edge_payload", "edge_outcome", "invalid", "child_visited", "child_prior",
        "child_value", "child_payload", "child_outcome", "child_to_play")]


class SynthParams(C.Structure):
    _fields_ = [
        ("seed_k0", C.c_uint32), ("seed_k1", C.c_uint32), ("num_actions", C.c_int32),
        ("legal_prob", C.c_float), ("terminal_prob", C.c_float),
        ("degenerate_lane_prob", C.c_float), ("degenerate_alpha", C.c_float),
        ("logc_mean", C.c_float), ("logc_std", C.c_float),
        ("logc_min", C.c_float), ("logc_max", C.c_float),
    ]


def _key(key) -> tuple[int, int]:
    k = np.asarray(key, dtype=np.uint32).reshape(2)
    return int(k[0]), int(k[1])


# --------------------------------------------------------------------------
# jax.random primitives
# --------------------------------------------------------------------------

def threefry(key, count) -> np.ndarray:
    out = np.zeros(2, np.uint32)
    k0, k1 = _key(key)
    c = np.asarray(count, dtype=np.uint32).reshape(2)
    lib().or_threefry(C.c_uint32(k0), C.c_uint32(k1), C.c_uint32(int(c[0])), C.c_uint32(int(c[1])), _p(out))
    return out


def random_bits(key, n: int) -> np.ndarray:
    out = np.zeros(n, np.uint32)
    k0, k1 = _key(key)
    lib().or_random_bits(C.c_uint32(k0), C.c_uint32(k1), C.c_uint64(n), _p(out))
    return out


def uniform(key, n: int, lo: float = 0.0, hi: float = 1.0) -> np.ndarray:
    out = np.zeros(n, np.float32)
    k0, k1 = _key(key)
    lib().or_uniform(C.c_uint32(k0), C.c_uint32(k1), C.c_uint64(n), C.c_float(lo), C.c_float(hi), _p(out))
    return out


def normal(key, n: int) -> np.ndarray:
    out = np.zeros(n, np.float32)
    k0, k1 = _key(key)
    lib().or_normal(C.c_uint32(k0), C.c_uint32(k1), C.c_uint64(n), _p(out))
    return out


MATH_FNS = {"log": 0, "exp": 1, "log1p": 2, "expm1": 3, "lgamma": 4, "betaln": 5,
            "erfinv": 6, "sinh": 7, "asinh": 8, "softplus": 9}


def math(fn: str, x, y=None) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32).ravel()
    y = np.ascontiguousarray(np.zeros_like(x) if y is None else y, dtype=np.float32).ravel()
    out = np.zeros_like(x)
    lib().or_math(C.c_int(MATH_FNS[fn]), _p(x), _p(y), C.c_int(x.size), _p(out))
    return out


# --------------------------------------------------------------------------
# estimators
# --------------------------------------------------------------------------

class PrefixResult(NamedTuple):
    policy: np.ndarray
    raw_policy: np.ndarray
    raw_mass: np.ndarray
    normalization_error: np.ndarray
    finite: np.ndarray
    grid_half_range: np.ndarray
    tail_range_clipped: np.ndarray
    density_log_integral: np.ndarray
    fallback_interval_count: np.ndarray


def prefix_params(half_width=10, tail_scale=8.0, min_half_range=6.0, max_half_range=11.0) -> PrefixParams:
    return PrefixParams(int(half_width), float(tail_scale), float(min_half_range), float(max_half_range))


def prefix_cdf(alpha, invalid, categorical_outcome=None, *, half_width=10, tail_scale=8.0,
               min_half_range=6.0, max_half_range=11.0) -> PrefixResult:
    alpha = np.ascontiguousarray(alpha, np.float32)
    B, A, _ = alpha.shape
    invalid = np.ascontiguousarray(invalid, np.uint8)
    if categorical_outcome is None:
        categorical_outcome = np.full((B, A), NO_OUTCOME, np.int8)
    cat = np.ascontiguousarray(categorical_outcome, np.int8)
    r = PrefixResult(
        np.zeros((B, A), np.float32), np.zeros((B, A), np.float32), np.zeros(B, np.float32),
        np.zeros(B, np.float32), np.zeros(B, np.uint8), np.zeros(B, np.float32),
        np.zeros(B, np.uint8), np.zeros((B, A), np.float32), np.zeros(B, np.int32))
    out = PrefixOut(*[_p(x) for x in r])
    prm = prefix_params(half_width, tail_scale, min_half_range, max_half_range)
    lib().or_prefix_cdf(_p(alpha), _p(invalid), _p(cat), C.c_int(B), C.c_int(A), C.byref(prm), C.byref(out))
    return r._replace(finite=r.finite.astype(bool), tail_range_clipped=r.tail_range_clipped.astype(bool))


def posterior_best_policy(key, alpha, invalid, num_samples: int, categorical_outcome=None) -> np.ndarray:
    alpha = np.ascontiguousarray(alpha, np.float32)
    B, A, _ = alpha.shape
    invalid = np.ascontiguousarray(invalid, np.uint8)
    cat = None if categorical_outcome is None else np.ascontiguousarray(categorical_outcome, np.int8)
    out = np.zeros((B, A), np.float32)
    lib().or_posterior_best_policy(_skey(key), _p(alpha), _p(invalid), _p(cat), C.c_int(B), C.c_int(A),
                                   C.c_int(num_samples), _p(out))
    return out


def thompson_sample(key, alpha, invalid, categorical_outcome=None) -> np.ndarray:
    alpha = np.ascontiguousarray(alpha, np.float32)
    B, A, _ = alpha.shape
    invalid = np.ascontiguousarray(invalid, np.uint8)
    cat = None if categorical_outcome is None else np.ascontiguousarray(categorical_outcome, np.int8)
    out = np.zeros(B, np.int32)
    lib().or_thompson_sample(_skey(key), _p(alpha), _p(invalid), _p(cat), C.c_int(B), C.c_int(A), _p(out))
    return out


def sample_dirichlet(key, alpha) -> np.ndarray:
    alpha = np.ascontiguousarray(alpha, np.float32).reshape(-1, 2)
    out = np.zeros_like(alpha)
    lib().or_sample_dirichlet(_skey(key), _p(alpha), C.c_int(alpha.shape[0]), _p(out))
    return out


class _SKey(C.Structure):
    _fields_ = [("k0", C.c_uint32), ("k1", C.c_uint32)]


def _skey(key) -> _SKey:
    k0, k1 = _key(key)
    return _SKey(k0, k1)


# --------------------------------------------------------------------------
# update rules
# --------------------------------------------------------------------------

@dataclasses.dataclass(frozen=True)
class Rule:
    """Static parameters of ``update_posterior`` / ``update_posterior_prefix_cdf``."""

    prefix_cdf: bool = True
    kappa: float = 4.0
    samples: int = 32
    half_width: int = 10
    tail_scale: float = 8.0
    min_half_range: float = 6.0
    max_half_range: float = 11.0
    density_tol: float = 0.01

    def params(self) -> UpdateParams:
        return UpdateParams(
            1 if self.prefix_cdf else 0, 1 if self.kappa >= 1.0 else 0,
            float(np.float32(1.0 / self.kappa)), float(np.float32(min(self.kappa, 1.0))), int(self.samples),
            prefix_params(self.half_width, self.tail_scale, self.min_half_range, self.max_half_range),
            float(np.float32(self.density_tol)))


CONTEXT_FIELDS = {
    "active": np.uint8, "leaf_active": np.uint8, "leaf_action": np.int32, "leaf_value": np.float32,
    "leaf_to_play": np.int32, "node_to_play": np.int32, "node_payload": np.int32,
    "value_prior": np.float32, "value_alpha": np.float32, "edge_alpha": np.float32,
    "edge_payload": np.int32, "edge_outcome": np.int8, "invalid": np.uint8,
    "child_visited": np.uint8, "child_prior": np.float32, "child_value": np.float32,
    "child_payload": np.int32, "child_outcome": np.int8, "child_to_play": np.int32,
}


def update_posterior(key, context: dict, rule: Rule):
    """Apply one repair rule to explicit contexts.

    ``context`` holds the ``NodeView`` / ``ChildrenView`` / ``LeafView`` fields
    (names of ``CONTEXT_FIELDS``) as arrays with a leading batch axis.
    Returns (edge_alpha, edge_payload, value_alpha, unsafe).
    """
    arrs = {k: np.ascontiguousarray(context[k], dt) for k, dt in CONTEXT_FIELDS.items()}
    B, A = arrs["edge_payload"].shape
    soa = ContextSoA(*[_p(arrs[k]) for k in CONTEXT_FIELDS])
    ea = np.zeros((B, A, 2), np.float32)
    ep = np.zeros((B, A), np.int32)
    va = np.zeros((B, 2), np.float32)
    unsafe = np.zeros(B, np.uint8)
    k0, k1 = _key(key)
    prm = rule.params()
    lib().or_update_posterior_soa(C.c_uint32(k0), C.c_uint32(k1), C.byref(soa), C.c_int(B), C.c_int(A),
                                  C.byref(prm), _p(ea), _p(ep), _p(va), _p(unsafe))
    return ea, ep, va, unsafe.astype(bool)


# --------------------------------------------------------------------------
# tree
# --------------------------------------------------------------------------

@dataclasses.dataclass
class Tree:
    """Numpy mirror of ``dirichlet_mctx.tree.Tree`` (binary outcomes)."""

    parents: np.ndarray
    children_index: np.ndarray
    node_to_play: np.ndarray
    node_categorical_outcome: np.ndarray
    node_payload: np.ndarray
    edge_categorical_outcome: np.ndarray
    edge_payload: np.ndarray
    node_value_priors: np.ndarray
    node_value_alpha: np.ndarray
    edge_alpha: np.ndarray
    invalid_actions: np.ndarray
    embeddings: np.ndarray
    lane_offset: int = 0
    total_batch: int = 0

    @classmethod
    def empty(cls, B: int, num_nodes: int, A: int, emb_bytes: int = 0) -> "Tree":
        return cls(
            np.zeros((B, num_nodes), np.int32), np.zeros((B, num_nodes, A), np.int32),
            np.zeros((B, num_nodes), np.int32), np.zeros((B, num_nodes), np.int8),
            np.zeros((B, num_nodes), np.int32), np.zeros((B, num_nodes, A), np.int8),
            np.zeros((B, num_nodes, A), np.int32), np.zeros((B, num_nodes, 2), np.float32),
            np.zeros((B, num_nodes, 2), np.float32), np.zeros((B, num_nodes, A, 2), np.float32),
            np.zeros((B, num_nodes, A), np.uint8), np.zeros((B, num_nodes, max(emb_bytes, 1)), np.uint8))

    @property
    def dims(self):
        B, Cn, A = self.children_index.shape
        return B, Cn, A

    def struct(self) -> TreeStruct:
        B, Cn, A = self.dims
        emb = self.embeddings.shape[-1] if self.embeddings.shape[-1] > 1 else 0
        return TreeStruct(B, Cn, A, emb, *[_p(x) for x in (
            self.parents, self.children_index, self.node_to_play, self.node_categorical_outcome,
            self.node_payload, self.edge_categorical_outcome, self.edge_payload,
            self.node_value_priors, self.node_value_alpha, self.edge_alpha,
            self.invalid_actions, self.embeddings)], self.lane_offset, self.total_batch)

    def summary(self) -> dict:
        B, _, A = self.dims
        out = dict(visit_counts=np.zeros((B, A), np.float32), alpha=np.zeros((B, A, 2), np.float32),
                   value_alpha=np.zeros((B, 2), np.float32), q_categorical_outcome=np.zeros((B, A), np.int8),
                   q_categorical_distance=np.zeros((B, A), np.int32),
                   v_categorical_outcome=np.zeros(B, np.int8), v_categorical_distance=np.zeros(B, np.int32))
        s = self.struct()
        lib().or_summary(C.byref(s), *[_p(out[k]) for k in (
            "visit_counts", "alpha", "value_alpha", "q_categorical_outcome", "q_categorical_distance",
            "v_categorical_outcome", "v_categorical_distance")])
        return out


def tree_init(root_value, root_action_values, root_invalid, root_terminal, root_to_play, num_simulations,
              root_embedding=None) -> Tree:
    root_action_values = np.ascontiguousarray(root_action_values, np.float32)
    B, A, _ = root_action_values.shape
    emb_bytes = 0 if root_embedding is None else int(np.asarray(root_embedding).reshape(B, -1).shape[1])
    t = Tree.empty(B, num_simulations + 1, A, emb_bytes)
    s = t.struct()
    emb = None if root_embedding is None else np.ascontiguousarray(root_embedding, np.uint8).reshape(B, -1)
    lib().or_tree_init(C.byref(s), _p(np.ascontiguousarray(root_value, np.float32)), _p(root_action_values),
                       _p(np.ascontiguousarray(root_invalid, np.uint8)),
                       _p(np.ascontiguousarray(root_terminal, np.int8)),
                       _p(np.ascontiguousarray(root_to_play, np.int32)), _p(emb))
    return t


def simulate(tree: Tree, simulate_key, max_depth: int):
    B = tree.dims[0]
    parent = np.zeros(B, np.int32)
    action = np.zeros(B, np.int32)
    active = np.zeros(B, np.uint8)
    s = tree.struct()
    lib().or_simulate(C.byref(s), _skey(simulate_key), C.c_int(max_depth), _p(parent), _p(action), _p(active))
    return parent, action, active.astype(bool)


def expand(tree: Tree, new_node: int, parent, action, active, step: dict, child_embedding=None):
    s = tree.struct()
    emb = None if child_embedding is None else np.ascontiguousarray(child_embedding, np.uint8)
    lib().or_expand(C.byref(s), C.c_int(new_node), _p(np.ascontiguousarray(parent, np.int32)),
                    _p(np.ascontiguousarray(action, np.int32)), _p(np.ascontiguousarray(active, np.uint8)),
                    _p(np.ascontiguousarray(step["value"], np.float32)),
                    _p(np.ascontiguousarray(step["action_values"], np.float32)),
                    _p(np.ascontiguousarray(step["invalid_actions"], np.uint8)),
                    _p(np.ascontiguousarray(step["terminal_outcome"], np.int8)),
                    _p(np.ascontiguousarray(step["to_play"], np.int32)), _p(emb))


def backward(tree: Tree, backward_key, parent, action, active, step_value, step_to_play, rule: Rule) -> int:
    s = tree.struct()
    prm = rule.params()
    lib().or_backward.restype = C.c_long
    return int(lib().or_backward(
        C.byref(s), _skey(backward_key), _p(np.ascontiguousarray(parent, np.int32)),
        _p(np.ascontiguousarray(action, np.int32)), _p(np.ascontiguousarray(active, np.uint8)),
        _p(np.ascontiguousarray(step_value, np.float32)), _p(np.ascontiguousarray(step_to_play, np.int32)),
        C.byref(prm)))


def categorize_and_publish(tree: Tree, node, active):
    s = tree.struct()
    lib().or_categorize_and_publish(C.byref(s), _p(np.ascontiguousarray(node, np.int32)),
                                    _p(np.ascontiguousarray(active, np.uint8)))


def root_policy(tree: Tree, policy_key, invalid, policy_samples: int):
    B, _, A = tree.dims
    w = np.zeros((B, A), np.float32)
    act = np.zeros(B, np.int32)
    s = tree.struct()
    lib().or_root_policy(C.byref(s), _skey(policy_key), _p(np.ascontiguousarray(invalid, np.uint8)),
                         C.c_int(policy_samples), _p(w), _p(act))
    return w, act


# --------------------------------------------------------------------------
# jax.random key schedule (host side, via the C threefry)
# --------------------------------------------------------------------------

def split(key, n: int = 2) -> np.ndarray:
    return np.stack([threefry(key, (0, i)) for i in range(n)])


def fold_in(key, d: int) -> np.ndarray:
    return threefry(key, (0, d))


def PRNGKey(seed: int) -> np.ndarray:
    return np.array([0, seed & 0xFFFFFFFF], np.uint32)


# --------------------------------------------------------------------------
# full search: Python-driven loop (any recurrent fn) and the C synthetic loop
# --------------------------------------------------------------------------

class PolicyOutput(NamedTuple):
    action: np.ndarray
    action_weights: np.ndarray
    search_tree: Tree
    unsafe_updates: int


def dirichlet_thompson_policy(rng_key, *, root: dict, recurrent_fn: Callable, num_simulations: int,
                              invalid_actions=None, rule: Rule = Rule(prefix_cdf=False), max_depth=None,
                              policy_samples: int = 32, lane_offset: int = 0,
                              total_batch: int = 0) -> PolicyOutput:
    """policies.py:17-48 + search.py:189-251 driven from Python.

    ``root``: dict with value [B,2], action_values [B,A,2], terminal_outcome,
    to_play, prior_logits and optionally embedding [B,E] (uint8 rows).
    ``recurrent_fn(action, parent_embedding) -> (step dict, child_embedding)``.
    The B lanes may be lanes [lane_offset, lane_offset + B) of a batch of
    ``total_batch`` lanes: lane-indexed and batch-wide random streams then
    use the lanes' places in that batch (bit-identical to the same lanes of
    a full run).
    """
    if max_depth is None:
        max_depth = num_simulations
    max_depth = max(1, int(max_depth))
    if invalid_actions is None:
        invalid_actions = ~np.isfinite(np.asarray(root["prior_logits"], np.float32))
    invalid_actions = np.asarray(invalid_actions, bool)
    search_key, policy_key = split(rng_key)
    emb = root.get("embedding")
    tree = tree_init(root["value"], root["action_values"], invalid_actions, root["terminal_outcome"],
                     root["to_play"], num_simulations, emb)
    tree.lane_offset, tree.total_batch = int(lane_offset), int(total_batch)
    unsafe = 0
    key = search_key
    B = tree.dims[0]
    for i in range(num_simulations):
        key, sim_key, _exp_key, bwd_key = split(key, 4)
        parent, action, active = simulate(tree, sim_key, max_depth)
        p = np.where(active, parent, 0)
        a = np.where(active, action, 0).astype(np.int32)
        parent_emb = tree.embeddings[np.arange(B), p]
        step, child_emb = recurrent_fn(a, parent_emb)
        expand(tree, i + 1, parent, action, active, step, child_emb)
        unsafe += backward(tree, bwd_key, parent, action, active, step["value"], step["to_play"], rule)
    w, act = root_policy(tree, policy_key, invalid_actions, max(1, policy_samples))
    return PolicyOutput(act, w, tree, unsafe)


def synth_params(seed: int = 0, num_actions: int = 82, legal_prob: float = 0.7, terminal_prob: float = 0.0,
                 degenerate_lane_prob: float = 0.01, degenerate_alpha: float = 1e-3, logc_mean: float = 0.5,
                 logc_std: float = 1.0, logc_min: float = -4.0, logc_max: float = 6.0) -> SynthParams:
    k = PRNGKey(seed)
    return SynthParams(int(k[0]), int(k[1]), num_actions, legal_prob, terminal_prob, degenerate_lane_prob,
                       degenerate_alpha, logc_mean, logc_std, logc_min, logc_max)


def synthetic_root(env: SynthParams, B: int) -> dict:
    A = env.num_actions
    out = dict(prior_logits=np.zeros((B, A), np.float32), value=np.zeros((B, 2), np.float32),
               action_values=np.zeros((B, A, 2), np.float32), invalid_actions=np.zeros((B, A), np.uint8),
               terminal_outcome=np.zeros(B, np.int8), to_play=np.zeros(B, np.int32),
               embedding=np.zeros((B, 16), np.uint8))
    lib().or_synthetic_root(C.byref(env), C.c_int(B), C.c_int(0), *[_p(out[k]) for k in (
        "prior_logits", "value", "action_values", "invalid_actions", "terminal_outcome", "to_play",
        "embedding")])
    out["invalid_actions"] = out["invalid_actions"].astype(bool)
    return out


def synthetic_recurrent(env: SynthParams, action, parent_embedding):
    action = np.ascontiguousarray(action, np.int32)
    B = action.shape[0]
    A = env.num_actions
    step = dict(value=np.zeros((B, 2), np.float32), action_values=np.zeros((B, A, 2), np.float32),
                invalid_actions=np.zeros((B, A), np.uint8), terminal_outcome=np.zeros(B, np.int8),
                to_play=np.zeros(B, np.int32))
    child = np.zeros((B, 16), np.uint8)
    lib().or_synthetic_recurrent(C.byref(env), C.c_int(B), C.c_int(0), _p(action),
                                 _p(np.ascontiguousarray(parent_embedding, np.uint8)),
                                 *[_p(step[k]) for k in ("value", "action_values", "invalid_actions",
                                                         "terminal_outcome", "to_play")], _p(child))
    return step, child


def search_synthetic(env: SynthParams, B: int, rng_key, num_simulations: int, rule: Rule,
                     max_depth=None, policy_samples: int = 32, lanes: tuple[int, int] | None = None
                     ) -> PolicyOutput:
    """The whole search on the synthetic game, loop in C.  ``lanes=(lo, hi)``
    runs only lanes [lo, hi) of the B-lane batch (bit-identical to the same
    lanes of a full run); the returned arrays then hold hi - lo lanes."""
    if max_depth is None:
        max_depth = num_simulations
    A = env.num_actions
    lo, hi = (0, B) if lanes is None else lanes
    tree = Tree.empty(hi - lo, num_simulations + 1, A, 16)
    tree.lane_offset, tree.total_batch = lo, B
    B = hi - lo
    w = np.zeros((B, A), np.float32)
    act = np.zeros(B, np.int32)
    s = tree.struct()
    prm = rule.params()
    k0, k1 = _key(rng_key)
    lib().or_search_synthetic.restype = C.c_long
    unsafe = lib().or_search_synthetic(C.byref(env), C.byref(s), C.c_uint32(k0), C.c_uint32(k1),
                                       C.c_int(num_simulations), C.c_int(max(1, int(max_depth))), C.byref(prm),
                                       C.c_int(max(1, policy_samples)), None, _p(w), _p(act))
    return PolicyOutput(act, w, tree, int(unsafe))


def root_readout(native, summary: dict, legal, *, search_evidence: bool, temperature: float, rule: Rule):
    """play_search._dirichlet_root_policy_readout for the numerical update."""
    native = np.ascontiguousarray(native, np.float32)
    B, A = native.shape
    target = np.zeros((B, A), np.float32)
    accepted = np.zeros(B, np.uint8)
    prm = prefix_params(rule.half_width, rule.tail_scale, rule.min_half_range, rule.max_half_range)
    lib().or_root_readout(
        C.c_int(B), C.c_int(A), _p(native), _p(np.ascontiguousarray(summary["visit_counts"], np.float32)),
        _p(np.ascontiguousarray(summary["alpha"], np.float32)),
        _p(np.ascontiguousarray(summary["q_categorical_outcome"], np.int8)),
        _p(np.ascontiguousarray(summary["q_categorical_distance"], np.int32)),
        _p(np.ascontiguousarray(summary["v_categorical_outcome"], np.int8)),
        _p(np.ascontiguousarray(legal, np.uint8)), C.c_int(1 if search_evidence else 0),
        C.c_float(temperature), C.byref(prm), C.c_float(0.01), _p(target), _p(accepted))
    return target, accepted.astype(bool)


# --------------------------------------------------------------------------
# action commitment
# --------------------------------------------------------------------------

TARGET_PAD, TARGET_DIRICHLET, TARGET_CATEGORICAL = 0, 1, 2


def pack_targets(summary: dict, policy_target, legal, search_action, action_set: int = 0,
                 reduction: int = 0) -> dict:
    """play_search.py:490-548 (_run_dirichlet_thompson_search's target
    packing) with dirichlet_q_search.py:119-182 (build_q_supervision).
    action_set 0: positive search evidence or solved, 1: positive posterior
    policy or solved; reduction 0: mean over selected state-action pairs,
    1: legacy source-weighted.  numpy in, numpy out; keys are the
    PosteriorTargets field names."""
    legal = np.asarray(legal, bool)
    policy_target = np.asarray(policy_target, np.float32)
    q_count = summary["visit_counts"][..., None]
    q_cat = summary["q_categorical_outcome"] != -1
    v_cat = summary["v_categorical_outcome"] != -1
    q_kind = np.where(legal, np.where(q_cat, TARGET_CATEGORICAL, TARGET_DIRICHLET), TARGET_PAD).astype(np.int8)
    v_kind = np.where(v_cat, TARGET_CATEGORICAL, TARGET_DIRICHLET).astype(np.int8)
    positive_evidence = q_count.sum(-1) > 0
    evidence_mass = (q_count.sum(-1) + np.zeros_like(policy_target)).astype(np.float32)
    source_selected, source_weight = ((positive_evidence, evidence_mass) if action_set == 0 else
                                      (policy_target > 0, policy_target))
    selected = legal & (source_selected | q_cat)
    if reduction == 0:
        pair_weight = selected.astype(np.float32)
    else:
        with np.errstate(invalid="ignore"):
            pair_weight = np.where(legal & q_cat, np.maximum(source_weight, np.float32(1.0)), source_weight)
        pair_weight = np.where(selected, pair_weight, np.float32(0.0)).astype(np.float32)
    return dict(
        policy=policy_target, alpha_q=summary["alpha"], alpha_v=summary["value_alpha"],
        mask=policy_target.sum(-1) > 0, q_supervision_selected=selected,
        q_supervision_pair_weight=pair_weight,
        q_positive_evidence_action=legal & positive_evidence, q_positive_policy_action=legal & (policy_target > 0),
        search_action=np.asarray(search_action, np.int32), q_target_kind=q_kind,
        q_target_weight=legal.astype(np.float32), q_target_outcome=summary["q_categorical_outcome"],
        q_target_distance=summary["q_categorical_distance"], v_target_kind=v_kind,
        v_target_weight=np.ones_like(summary["v_categorical_distance"], np.float32),
        v_target_outcome=summary["v_categorical_outcome"], v_target_distance=summary["v_categorical_distance"])


def commitment_policy(sampled, search_action, alpha, q_outcome, v_outcome, legal, evidence, *,
                      search_evidence: bool, numerical: bool, rule: Rule = Rule()) -> np.ndarray:
    """play_search._dirichlet_commitment_policy for given sampled (Monte
    Carlo) policies."""
    sampled = np.ascontiguousarray(sampled, np.float32)
    B, A = sampled.shape
    out = np.zeros((B, A), np.float32)
    prm = prefix_params(rule.half_width, rule.tail_scale, rule.min_half_range, rule.max_half_range)
    lib().or_commitment_policy(
        C.c_int(B), C.c_int(A), _p(sampled), _p(np.ascontiguousarray(search_action, np.int32)),
        _p(np.ascontiguousarray(alpha, np.float32)), _p(np.ascontiguousarray(q_outcome, np.int8)),
        _p(np.ascontiguousarray(v_outcome, np.int8)), _p(np.ascontiguousarray(legal, np.uint8)),
        _p(np.ascontiguousarray(evidence, np.uint8)), C.c_int(int(search_evidence)), C.c_int(int(numerical)),
        C.byref(prm), _p(out))
    return out


def commit_action(kind: str, key, policy, legal, temperature: float = 1.0) -> np.ndarray:
    """posterior_best_action (kind "argmax") / posterior_sample_action
    (kind "sample")."""
    policy = np.ascontiguousarray(policy, np.float32)
    B, A = policy.shape
    out = np.zeros(B, np.int32)
    k0, k1 = _key(key if key is not None else [0, 0])
    lib().or_commit_action(C.c_int(0 if kind == "argmax" else 1), C.c_uint32(k0), C.c_uint32(k1), _p(policy),
                           _p(np.ascontiguousarray(legal, np.uint8)), C.c_int(B), C.c_int(A),
                           C.c_float(temperature), _p(out))
    return out
