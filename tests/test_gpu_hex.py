"""CUDA Hex kernels against the Hex restatement, and Hex searches.

* random playouts: every step's record, observation, invalid row, terminal
  outcome, player, rewards and terminated flag, bit for bit;
* init and the seeded root sampler;
* a whole search on Hex with a deterministic evaluator: the CUDA path
  (HexGame's fused recurrent function) against the oracle's search driven
  with the Hex restatement, every tree field bit for bit;
* make_search on Hex with the tcgen05 tower as evaluator (the full step's
  pipeline at a small size): targets are well formed.
"""

import numpy as np
import pytest
import torch

from oracle import hex_ref as H

pytestmark = pytest.mark.gpu


def _playout_actions(rng, records):
    acts = []
    for rec in records:
        b = H.HexBoard.from_record(rec)
        empty = np.nonzero(b.cells == 0)[0]
        acts.append(int(rng.choice(empty)) if (len(empty) and not b.terminated) else 0)
    return np.array(acts, np.int32)


@pytest.mark.parametrize("size", [3, 5, 9, 11])
def test_step_matches_restatement_over_playouts(cuda, size):
    from scacchi_b200.hex import HexGame, hex_error, lane_keys
    from scacchi_b200 import random as R

    rng = np.random.default_rng(size)
    B = 96
    game = HexGame(size)
    keys = lane_keys(R.PRNGKey(size), B)
    state = game.init(keys)
    want = [H.init_state(size, k) for k in keys]
    assert np.array_equal(state.record.cpu().numpy(), np.stack([w.record() for w in want]))
    np.testing.assert_array_equal(state.observation.cpu().numpy(), np.stack([w.observation() for w in want]))
    np.testing.assert_array_equal(state.legal_action_mask.cpu().numpy(), np.stack([w.legal() for w in want]))
    np.testing.assert_array_equal(state.current_player.cpu().numpy(), [w.current_player() for w in want])
    assert not state.terminated.any() and not state.rewards.any()
    records = state.record.cpu().numpy()
    for _ in range(size * size + 2):
        acts = _playout_actions(rng, records)
        got = game.step(state, torch.from_numpy(acts).cuda())
        outs = [H.step_outputs(r, a) for r, a in zip(records, acts)]
        np.testing.assert_array_equal(got.record.cpu().numpy(), np.stack([o["record"] for o in outs]))
        np.testing.assert_array_equal(got.observation.cpu().numpy(), np.stack([o["observation"] for o in outs]))
        np.testing.assert_array_equal((~got.legal_action_mask).cpu().numpy(), np.stack([o["invalid"] for o in outs]))
        np.testing.assert_array_equal(got.current_player.cpu().numpy(), [o["to_play"] for o in outs])
        np.testing.assert_array_equal(got.rewards.cpu().numpy(), np.stack([o["rewards"] for o in outs]))
        np.testing.assert_array_equal(got.terminated.cpu().numpy(), [o["terminated"] for o in outs])
        # the fused recurrent outputs: terminal outcome aligned to the child
        term = torch.empty(B, dtype=torch.int8, device="cuda")
        from scacchi_b200 import _lib
        from scacchi_b200.dirichlet_mctx.tree import ptr, stream_handle
        nxt = torch.empty_like(state.record)
        _lib.check(_lib.lib().scacchi_hex_step(B, ptr(state.record), ptr(torch.from_numpy(acts).cuda()), ptr(nxt),
                                               None, None, ptr(term), None, None, None,
                                               stream_handle(torch.device("cuda"))), "hex_step")
        np.testing.assert_array_equal(term.cpu().numpy(), [o["terminal"] for o in outs])
        state, records = got, got.record.cpu().numpy()
    assert records[:, 34].all()  # every playout ended
    assert hex_error() == 0


def test_random_roots_match_restatement(cuda):
    from scacchi_b200.hex import HexGame
    from scacchi_b200 import random as R

    key = R.PRNGKey(11)
    got = HexGame(9).random_roots(200, key, 0, 20)
    want = np.stack([H.random_root(9, np.asarray(key, np.uint32), b, 0, 20).record() for b in range(200)])
    np.testing.assert_array_equal(got.record.cpu().numpy(), want)
    obs = np.stack([H.HexBoard.from_record(r).observation() for r in want])
    np.testing.assert_array_equal(got.observation.cpu().numpy(), obs)


def toy_evaluator_np(obs: np.ndarray):
    """A deterministic float32 function of the observation (both sides run
    this same numpy code, so the search sees identical leaf values)."""
    f = np.float32
    B, s = obs.shape[0], obs.shape[1]
    own = obs[..., 0].reshape(B, -1)
    opp = obs[..., 1].reshape(B, -1)
    idx = np.arange(1, s * s + 1, dtype=f)
    h = (own * idx).sum(1, dtype=f) * f(0.37) + (opp * idx[::-1]).sum(1, dtype=f) * f(0.11) + obs[:, 0, 0, 2]
    phase = (h - np.floor(h)).astype(f)
    alpha_v = np.stack([f(0.5) + phase, f(1.5) - phase], -1).astype(f)
    a = np.arange(s * s + 1, dtype=f)[None]
    q = np.exp(np.sin(a * f(0.731) + phase[:, None] * f(6.0)).astype(f)).astype(f)
    alpha_q = np.stack([q, (f(2.0) / q).astype(f)], -1).astype(f)
    logits = np.zeros((B, s * s + 1), f)
    return logits, alpha_v, alpha_q


def test_hex_search_matches_oracle_search(cuda):
    from oracle import oracle as O
    from scacchi_b200 import dirichlet_mctx as dm
    from scacchi_b200 import random as R
    from scacchi_b200.dirichlet_mctx.posterior_updates import update_posterior_prefix_cdf
    from scacchi_b200.hex import HexGame
    from scacchi_b200.play_search import EvaluatorOutput
    import functools

    size, B, N = 5, 32, 40
    game = HexGame(size)
    root_key = R.PRNGKey(2)
    state = game.random_roots(B, root_key, 10, 16)  # crowded boards: wins within reach
    records = state.record.cpu().numpy()

    def evaluator(obs):
        lg, av, aq = toy_evaluator_np(obs.cpu().numpy())
        return EvaluatorOutput(logits=torch.from_numpy(lg).cuda(), alpha_v=torch.from_numpy(av).cuda(),
                               alpha_q=torch.from_numpy(aq).cuda())

    lg, av, aq = toy_evaluator_np(state.observation.cpu().numpy())
    inv = ~state.legal_action_mask.cpu().numpy()
    # root terminal outcome from the player to move's reward (play_search.py:457-462)
    boards = [H.HexBoard.from_record(r) for r in records]
    root_term = np.array([(int(b.rewards()[b.current_player()]) + 1) // 2 if b.terminated else -1 for b in boards],
                         np.int8)
    root = dm.RootFnOutput(prior_logits=torch.from_numpy(np.where(inv, -np.inf, lg).astype(np.float32)).cuda(),
                           value=torch.from_numpy(av).cuda(), action_values=torch.from_numpy(aq).cuda(),
                           embedding=state.record, terminal_outcome=torch.from_numpy(root_term).cuda(),
                           to_play=state.current_player)
    rule = functools.partial(update_posterior_prefix_cdf, kappa=1.0, fallback_policy_samples=8)
    key = R.PRNGKey(9)
    out = dm.dirichlet_thompson_policy((), key, root=root, recurrent_fn=game.native_recurrent_fn(evaluator),
                                       num_simulations=N, invalid_actions=torch.from_numpy(inv).cuda(),
                                       posterior_update=rule, max_depth=N, policy_samples=8)
    torch.cuda.synchronize()

    def recurrent(actions, parent_emb):
        outs = [H.step_outputs(r, a) for r, a in zip(parent_emb, actions)]
        _, v, q = toy_evaluator_np(np.stack([o["observation"] for o in outs]))
        step = dict(value=v, action_values=q, invalid_actions=np.stack([o["invalid"] for o in outs]),
                    terminal_outcome=np.array([o["terminal"] for o in outs], np.int8),
                    to_play=np.array([o["to_play"] for o in outs], np.int32))
        return step, np.stack([o["record"] for o in outs])

    want = O.dirichlet_thompson_policy(
        np.asarray(key, np.uint32),
        root=dict(prior_logits=np.where(inv, -np.inf, lg).astype(np.float32), value=av, action_values=aq,
                  terminal_outcome=root_term, to_play=state.current_player.cpu().numpy(),
                  embedding=records),
        recurrent_fn=recurrent, num_simulations=N, invalid_actions=inv,
        rule=O.Rule(prefix_cdf=True, kappa=1.0, samples=8), max_depth=N, policy_samples=8)
    fields = ("parents", "children_index", "node_to_play", "node_categorical_outcome", "node_payload",
              "edge_categorical_outcome", "edge_payload", "node_value_priors", "node_value_alpha", "edge_alpha",
              "invalid_actions")
    for f in fields:
        a = getattr(out.search_tree, f).cpu().numpy()
        b = getattr(want.search_tree, f)
        assert np.array_equal(a.astype(b.dtype), b), f
    # node states: the 48-byte records of every expanded node
    parents = want.search_tree.parents
    expanded = parents >= 0
    expanded[:, 0] = True
    emb = out.search_tree.embedding_.cpu().numpy()[..., :H.RECORD_BYTES]
    assert np.array_equal(emb[expanded], want.search_tree.embeddings[expanded])
    assert np.array_equal(out.action_weights.cpu().numpy(), want.action_weights)
    assert np.array_equal(out.action.cpu().numpy(), want.action)
    # terminal certificates appear on this small board
    assert (want.search_tree.node_categorical_outcome >= 0).any()


def test_make_search_on_hex_with_tower(cuda):
    from scacchi_b200 import random as R
    from scacchi_b200.hex import HexGame
    from scacchi_b200.network import AZDirichletNet, init_params
    from scacchi_b200.play_search import make_evaluator, make_search
    from scacchi_b200.types import (DirichletThompsonSearchConfig, NumericalPosteriorUpdateConfig,
                                    PosteriorUpdateConfig, PosteriorUpdateKind, RootPolicySupport)

    B, N = 64, 16
    game = HexGame(9)
    net = AZDirichletNet(init_params(0, he_all_layers=True, block_gain=0.5))
    cfg = DirichletThompsonSearchConfig(
        num_simulations=N, max_depth=N, root_policy_support=RootPolicySupport.search_evidence,
        posterior_update=PosteriorUpdateConfig(kind=PosteriorUpdateKind.numerical,
                                               numerical=NumericalPosteriorUpdateConfig(
                                                   kappa=1.0, fallback_policy_samples=8)))
    search = make_search(game, make_evaluator(net), cfg)
    state = game.random_roots(B, R.PRNGKey(4), 0, 20)
    t = search(state, R.PRNGKey(5))
    torch.cuda.synchronize()
    legal = state.legal_action_mask
    pol = t.prediction.policy
    assert torch.allclose(pol.sum(-1), torch.ones(B, device="cuda"), atol=1e-5)
    assert not (pol[~legal] > 0).any()
    act = t.metadata.search_action.long()
    assert legal[torch.arange(B, device="cuda"), act].all()
    assert torch.isfinite(t.prediction.alpha_q).all() and torch.isfinite(t.prediction.alpha_v).all()
