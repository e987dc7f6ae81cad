"""Action commitment on the CUDA path: kernels against the oracle bit for
bit, and the reference's player tests (tests/test_play.py:368-470,
675-733 of the reference) on its toy environment."""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _t(x, dt):
    return torch.as_tensor(np.asarray(x)).cuda().to(dt)


@pytest.mark.parametrize("A", [5, 82])
@pytest.mark.parametrize("temperature", [1.0, 1.0 / 3.0, 2.5])
def test_commit_action_matches_oracle(cuda, A, temperature):
    from oracle import oracle as O
    from scacchi_b200.play_search import posterior_best_action, posterior_sample_action

    rng = np.random.default_rng(A + int(temperature * 10))
    B = 301
    policy = rng.dirichlet(np.ones(A), B).astype(np.float32)
    policy[rng.uniform(size=(B, A)) < 0.3] = 0.0
    policy[:5] = 0.0  # no positive action: the legal fallback
    legal = rng.uniform(size=(B, A)) < 0.8
    legal[7] = False
    key = np.array([123, 456], np.uint32)
    got = posterior_sample_action(key, _t(policy, torch.float32), _t(legal, torch.bool), temperature)
    assert np.array_equal(got.cpu().numpy(), O.commit_action("sample", key, policy, legal, temperature))
    got = posterior_best_action(_t(policy, torch.float32), _t(legal, torch.bool))
    assert np.array_equal(got.cpu().numpy(), O.commit_action("argmax", None, policy, legal))


@pytest.mark.parametrize("numerical", [False, True])
@pytest.mark.parametrize("search_evidence", [False, True])
def test_commitment_policy_matches_oracle(cuda, numerical, search_evidence):
    from oracle import oracle as O
    from scacchi_b200 import _lib
    from scacchi_b200.dirichlet_mctx.tree import ptr, stream_handle

    rng = np.random.default_rng(10 * numerical + search_evidence)
    B, A = 97, 82
    alpha = np.exp(rng.uniform(-4, 5, (B, A, 2))).astype(np.float32)
    alpha[3] = 1e-3
    sampled = rng.dirichlet(np.ones(A), B).astype(np.float32)
    sampled[rng.uniform(size=(B, A)) < 0.5] = 0.0
    legal = rng.uniform(size=(B, A)) < 0.8
    evidence = rng.uniform(size=(B, A)) < 0.3
    q_out = np.where(rng.uniform(size=(B, A)) < 0.05, rng.integers(0, 2, (B, A)), -1).astype(np.int8)
    v_out = np.where(rng.uniform(size=B) < 0.1, rng.integers(0, 2, B), -1).astype(np.int8)
    action = rng.integers(0, A, B).astype(np.int32)
    want = O.commitment_policy(sampled, action, alpha, q_out, v_out, legal, evidence,
                               search_evidence=search_evidence, numerical=numerical)
    out = torch.empty((B, A), dtype=torch.float32, device="cuda")
    args = [_t(sampled, torch.float32), _t(action, torch.int32), _t(alpha, torch.float32), _t(q_out, torch.int8),
            _t(v_out, torch.int8), _t(legal, torch.uint8), _t(evidence, torch.uint8)]
    _lib.check(_lib.lib().scacchi_commitment_policy(B, A, *[ptr(a) for a in args], int(search_evidence),
                                                    int(numerical), 10, 8.0, 6.0, 11.0, ptr(out),
                                                    stream_handle(torch.device("cuda"))), "commitment_policy")
    assert np.array_equal(out.cpu().numpy(), want)


def _toy():
    import test_gpu_boundary as TB

    return TB


def _search_config(kind_update="numerical"):
    TB = _toy()
    return TB.config(0, kind_update, samples=8)


def test_search_player_composes_q21_action_with_cubic_sampling(cuda):
    # tests/test_play.py:367-415
    from scacchi_b200 import random as R
    from scacchi_b200.play_search import (dirichlet_commitment_policy, make_search, make_search_player,
                                          posterior_sample_action)
    from scacchi_b200.types import ActionCommitmentConfig, ActionCommitmentType, PosteriorUpdateKind

    TB = _toy()
    state = TB.toy_state()
    cfg = _search_config("numerical")
    player_key = R.PRNGKey(911)
    search_key, action_key = R.split(player_key)
    out = make_search(TB.ToyEnv(), TB.toy_evaluator, cfg)(state, search_key)
    policy_key, sample_key = R.split(action_key)
    policy = dirichlet_commitment_policy(out, state.legal_action_mask, policy_key, cfg.dirichlet_thompson,
                                         PosteriorUpdateKind.numerical)
    expected = posterior_sample_action(sample_key, policy, state.legal_action_mask, temperature=1.0 / 3.0)
    player = make_search_player(TB.ToyEnv(), TB.toy_evaluator, cfg, ActionCommitmentConfig(
        kind=ActionCommitmentType.posterior_sample, posterior_update=PosteriorUpdateKind.numerical,
        posterior_sample_temperature=1.0 / 3.0))
    assert torch.equal(player(state, player_key).action, expected)
    # the commitment policy itself: the Q21 readout on the support
    _check_commitment_policy(out, state, policy_key, policy, numerical=True)


def _check_commitment_policy(out, state, policy_key, policy, numerical):
    from oracle import oracle as O

    m = out.metadata
    legal = state.legal_action_mask.cpu().numpy()
    alpha = out.prediction.alpha_q.cpu().numpy()
    evidence = m.q_positive_evidence_action.cpu().numpy()
    q_out = m.q_target_outcome.cpu().numpy()
    support = legal & (evidence | (q_out != -1))
    support = np.where(support.any(-1, keepdims=True), support, legal)
    sampled = O.posterior_best_policy(policy_key, alpha, ~support, 8, q_out)
    want = O.commitment_policy(sampled, m.search_action.cpu().numpy(), alpha, q_out, m.v_target_outcome.cpu().numpy(),
                               legal, evidence, search_evidence=True, numerical=numerical)
    assert want.sum(-1).min() > 0.99  # a real distribution, not an empty support
    assert np.array_equal(policy.cpu().numpy(), want)


def test_action_commitment_can_select_a_different_posterior_update(cuda):
    # tests/test_play.py:418-470
    from scacchi_b200 import random as R
    from scacchi_b200.play_search import (dirichlet_commitment_policy, make_search, make_search_player,
                                          posterior_sample_action)
    from scacchi_b200.types import ActionCommitmentConfig, ActionCommitmentType, PosteriorUpdateKind

    TB = _toy()
    state = TB.toy_state()
    cfg = _search_config("numerical")
    commitment = ActionCommitmentConfig(kind=ActionCommitmentType.posterior_sample,
                                        posterior_update=PosteriorUpdateKind.monte_carlo)
    player_key = R.PRNGKey(913)
    search_key, action_key = R.split(player_key)
    out = make_search(TB.ToyEnv(), TB.toy_evaluator, cfg)(state, search_key)
    policy_key, sample_key = R.split(action_key)
    policy = dirichlet_commitment_policy(out, state.legal_action_mask, policy_key, cfg.dirichlet_thompson,
                                         PosteriorUpdateKind.monte_carlo)
    expected = posterior_sample_action(sample_key, policy, state.legal_action_mask)
    got = make_search_player(TB.ToyEnv(), TB.toy_evaluator, cfg, commitment)(state, player_key)
    assert torch.equal(got.action, expected)
    # the Monte Carlo commitment policy: the population over the support,
    # renormalised there (no Q21)
    _check_commitment_policy(out, state, policy_key, policy, numerical=False)


def test_unsafe_q21_action_update_uses_its_monte_carlo_fallback(cuda):
    # tests/test_play.py:675-733
    from scacchi_b200 import random as R
    from scacchi_b200.play_search import EvaluatorOutput, dirichlet_commitment_policy, make_search
    from scacchi_b200.types import PosteriorUpdateKind

    TB = _toy()
    state = TB.toy_state()

    def extreme_evaluator(obs):
        B = obs.shape[0]
        q = torch.tensor([[1e-8, 1.0], [1.0, 1e-8], [1.0, 1.0]], device="cuda")
        return EvaluatorOutput(logits=torch.zeros((B, 3), device="cuda"), alpha_v=torch.ones((B, 2), device="cuda"),
                               alpha_q=q.expand(B, 3, 2).contiguous())

    cfg = _search_config("numerical")
    out = make_search(TB.ToyEnv(), extreme_evaluator, cfg)(state, R.PRNGKey(92))
    key = R.PRNGKey(123)
    numerical = dirichlet_commitment_policy(out, state.legal_action_mask, key, cfg.dirichlet_thompson,
                                            PosteriorUpdateKind.numerical)
    native = dirichlet_commitment_policy(out, state.legal_action_mask, key, cfg.dirichlet_thompson,
                                         PosteriorUpdateKind.monte_carlo)
    assert torch.equal(numerical, native)
