"""Whole searches on the synthetic game: CUDA vs the oracle, bit for bit.

Small batches compare every tree field; the full isolated-search workload
(4096 lanes x 128 simulations, 82 actions) compares sampled lanes against
oracle runs of exactly those lanes, and checks size-independent invariants
over every lane.
"""

import functools

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TREE_FIELDS = ("parents", "children_index", "node_to_play", "node_categorical_outcome", "node_payload",
               "edge_categorical_outcome", "edge_payload", "node_value_priors", "node_value_alpha", "edge_alpha",
               "invalid_actions")


def run_cuda(B, N, prefix, terminal_prob, seed=0, key_seed=0, samples=8, kappa=1.0, native=True, lanes=None,
             max_depth=None, **env):
    from scacchi_b200 import dirichlet_mctx as dm
    from scacchi_b200 import random as R
    from scacchi_b200.synthetic import SyntheticGame, SyntheticGameConfig

    game = SyntheticGame(SyntheticGameConfig(seed=seed, terminal_prob=terminal_prob, **env))
    root = game.root(B)
    rule = (functools.partial(dm.update_posterior_prefix_cdf, kappa=kappa, fallback_policy_samples=samples)
            if prefix else functools.partial(dm.update_posterior, kappa=kappa, policy_samples=samples))
    rec = game if native else (lambda p, k, a, e: game(p, k, a, e))
    stats = torch.zeros(6, dtype=torch.int64, device="cuda")
    out = dm.dirichlet_thompson_policy((), R.PRNGKey(key_seed), root=root, recurrent_fn=rec, num_simulations=N,
                                       posterior_update=rule, max_depth=N if max_depth is None else max_depth,
                                       policy_samples=samples, stats=stats)
    torch.cuda.synchronize()
    return out, stats.cpu().numpy()


def run_oracle(B, N, prefix, terminal_prob, seed=0, key_seed=0, samples=8, kappa=1.0, lanes=None, max_depth=None,
               **env):
    from oracle import oracle as O

    env = O.synth_params(seed=seed, terminal_prob=terminal_prob, **env)
    return O.search_synthetic(env, B, O.PRNGKey(key_seed), N, O.Rule(prefix_cdf=prefix, kappa=kappa,
                                                                      samples=samples),
                              max_depth=N if max_depth is None else max_depth, policy_samples=samples, lanes=lanes)


def compare(out, want, lanes=slice(None)):
    tree = out.search_tree
    for f in TREE_FIELDS:
        a = getattr(tree, f)[lanes].cpu().numpy()
        b = getattr(want.search_tree, f)
        assert np.array_equal(a.astype(b.dtype), b), f
    assert np.array_equal(out.action_weights[lanes].cpu().numpy(), want.action_weights)
    assert np.array_equal(out.action[lanes].cpu().numpy(), want.action)


@pytest.mark.parametrize("prefix", [True, False], ids=["prefix_cdf", "mc"])
@pytest.mark.parametrize("terminal_prob", [0.0, 0.08])
def test_small_search_bit_exact(cuda, prefix, terminal_prob):
    out, stats = run_cuda(48, 24, prefix, terminal_prob)
    want = run_oracle(48, 24, prefix, terminal_prob)
    compare(out, want)
    if prefix:
        assert stats[2] == want.unsafe_updates


@pytest.mark.parametrize("num_actions", [20, 50, 120], ids=["one_warp", "two_warps", "four_warps"])
@pytest.mark.parametrize("prefix", [True, False], ids=["prefix_cdf", "mc"])
def test_action_counts_bit_exact(cuda, num_actions, prefix):
    # every CTA width; low concentrations make most variates take the
    # alpha < 1 augmentation and many first proposals fail
    env = dict(num_actions=num_actions, logc_mean=-1.0, logc_std=1.5)
    out, stats = run_cuda(24, 16, prefix, 0.05, seed=3, key_seed=4, **env)
    want = run_oracle(24, 16, prefix, 0.05, seed=3, key_seed=4, **env)
    compare(out, want)
    if prefix:
        assert stats[2] == want.unsafe_updates


@pytest.mark.parametrize("samples", [17, 40])
def test_population_chunks_bit_exact(cuda, samples):
    # several sample chunks, the last one partial
    out, _ = run_cuda(16, 12, False, 0.05, seed=6, key_seed=7, samples=samples)
    want = run_oracle(16, 12, False, 0.05, seed=6, key_seed=7, samples=samples)
    compare(out, want)


@pytest.mark.parametrize("B,N,max_depth", [(1, 1, 1), (1, 8, 1), (33, 3, 2), (2, 5, 5), (33, 1, None)],
                         ids=["one_lane_one_sim", "depth_one", "ragged_batch", "two_lanes", "one_sim"])
@pytest.mark.parametrize("prefix", [True, False], ids=["prefix_cdf", "mc"])
def test_edge_shapes_bit_exact(cuda, B, N, max_depth, prefix):
    """Batches of one lane and a batch that is not a multiple of 32, a
    single simulation, and a depth limit of one (search.py:192-197)."""
    out, _ = run_cuda(B, N, prefix, 0.1, seed=11, key_seed=12, max_depth=max_depth)
    want = run_oracle(B, N, prefix, 0.1, seed=11, key_seed=12, max_depth=max_depth)
    compare(out, want)


def test_python_loop_matches_native_loop(cuda):
    a, _ = run_cuda(32, 16, True, 0.05, native=True)
    b, _ = run_cuda(32, 16, True, 0.05, native=False)
    for f in TREE_FIELDS:
        assert torch.equal(getattr(a.search_tree, f), getattr(b.search_tree, f)), f
    assert torch.equal(a.action_weights, b.action_weights)


def test_full_size_sampled_lanes_and_invariants(cuda):
    """4096 lanes x 128 simulations (the isolated search-kernel workload)."""
    from scacchi_b200 import _lib

    B, N = 4096, 128
    out, stats = run_cuda(B, N, True, 0.0)
    assert _lib.device_error() == 0
    for lo, hi in ((0, 3), (1500, 1502), (4093, 4096)):
        want = run_oracle(B, N, True, 0.0, lanes=(lo, hi))
        compare(out, want, slice(lo, hi))
    tree = out.search_tree
    parents = tree.parents.cpu().numpy()
    children = tree.children_index.cpu().numpy()
    # every simulation expands at most one node per lane: node i+1's parent is < i+1
    idx = np.arange(N + 1)[None]
    expanded = parents >= 0
    assert np.all(parents[expanded] < np.broadcast_to(idx, parents.shape)[expanded])
    # child links are consistent with parent pointers
    b, n, a = np.nonzero(children >= 0)
    assert np.array_equal(parents[b, children[b, n, a]], n)
    # the policy target is a distribution over legal root actions
    w = out.action_weights.cpu().numpy()
    assert np.allclose(w.sum(-1), 1.0, atol=1e-5)
    assert stats[0] > 0 and stats[4] > 0


def test_search_boundary_targets(cuda):
    """make_search(...)(root_state, key) -> PosteriorTargets on the synthetic game."""
    from oracle import oracle as O
    from scacchi_b200 import random as R
    from scacchi_b200.play_search import make_search
    from scacchi_b200.synthetic import SyntheticGame, SyntheticGameConfig
    from scacchi_b200.types import (DirichletThompsonSearchConfig, NumericalPosteriorUpdateConfig,
                                    PosteriorUpdateConfig, PosteriorUpdateKind, RootPolicySupport)

    B, N = 64, 16
    game = SyntheticGame(SyntheticGameConfig(seed=3, terminal_prob=0.1))
    cfg = DirichletThompsonSearchConfig(
        num_simulations=N, max_depth=N, root_policy_support=RootPolicySupport.search_evidence,
        posterior_update=PosteriorUpdateConfig(kind=PosteriorUpdateKind.numerical,
                                               numerical=NumericalPosteriorUpdateConfig(
                                                   kappa=1.0, fallback_policy_samples=8)))
    search = make_search(game, game.evaluator, cfg)
    state = game.init(B)
    targets = search(state, R.PRNGKey(5))
    torch.cuda.synchronize()
    # oracle: the same search, then the root readout on the oracle summary
    env = O.synth_params(seed=3, terminal_prob=0.1)
    want = O.search_synthetic(env, B, O.PRNGKey(5), N, O.Rule(prefix_cdf=True, kappa=1.0, samples=8),
                              max_depth=N, policy_samples=8)
    s = want.search_tree.summary()
    legal = state.legal_action_mask.cpu().numpy()
    target, _ = O.root_readout(want.action_weights, s, legal, search_evidence=True, temperature=1.0,
                               rule=O.Rule(prefix_cdf=True))
    assert np.array_equal(targets.prediction.policy.cpu().numpy(), target)
    assert np.array_equal(targets.prediction.alpha_q.cpu().numpy(), s["alpha"])
    assert np.array_equal(targets.prediction.alpha_v.cpu().numpy(), s["value_alpha"])
    assert np.array_equal(targets.metadata.search_action.cpu().numpy(), want.action)
    assert np.array_equal(targets.metadata.q_target_distance.cpu().numpy(), s["q_categorical_distance"])


def test_fine_grid_search_uses_warp_kernel_bit_exact(cuda):
    """half_width 100 (Q = 201) does not fit the per-lane CTA's shared-memory
    matrices, so backward runs the warp-per-lane kernel; same results."""
    from oracle import oracle as O
    from scacchi_b200 import dirichlet_mctx as dm
    from scacchi_b200 import random as R
    from scacchi_b200.synthetic import SyntheticGame, SyntheticGameConfig

    B, N = 24, 12
    game = SyntheticGame(SyntheticGameConfig(seed=9, terminal_prob=0.05))
    rule = functools.partial(dm.update_posterior_prefix_cdf, kappa=1.0, half_width=100, fallback_policy_samples=4)
    out = dm.dirichlet_thompson_policy((), R.PRNGKey(2), root=game.root(B), recurrent_fn=game, num_simulations=N,
                                       posterior_update=rule, max_depth=N, policy_samples=4)
    want = O.search_synthetic(O.synth_params(seed=9, terminal_prob=0.05), B, O.PRNGKey(2), N,
                              O.Rule(prefix_cdf=True, kappa=1.0, samples=4, half_width=100), max_depth=N,
                              policy_samples=4)
    compare(out, want)
