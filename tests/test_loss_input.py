"""The loss-input restatement (oracle/loss_ref.py, the checker of the
scacchi_loss_input kernel; scacchi/loss.py:164-357) on CPU tensors, held to
the reference's assertions of tests/test_loss_masks.py:132-434.  The same
assertions run through the kernel in tests/test_gpu_targets.py."""

import torch

from oracle.loss_ref import make_compute_input_for_lossfn, trajectory_value_targets
from scacchi_b200.loss_input import TrainingLossConfig
from scacchi_b200.play import TrainingSamples
from scacchi_b200.play_search import (TARGET_CATEGORICAL, TARGET_DIRICHLET, PosteriorPrediction, PosteriorTargets,
                                      QSupervision, TargetMetadata)


def samples(obs, reward, terminated, action_weights, played_action, legal_action_mask, beta_q, beta_v, q_pair_weight,
            discount, search_loss_mask=None):
    return TrainingSamples(
        obs=obs, reward=reward, terminated=terminated, discount=discount,
        posterior=PosteriorTargets(
            prediction=PosteriorPrediction(policy=action_weights, alpha_v=beta_v, alpha_q=beta_q),
            metadata=TargetMetadata(mask=search_loss_mask,
                                    q_supervision=QSupervision(selected=q_pair_weight > 0, pair_weight=q_pair_weight))),
        played_action=played_action, legal_action_mask=legal_action_mask)


def test_preserves_root_legal_action_mask():
    # tests/test_loss_masks.py:132-212
    legal = torch.tensor([[[1, 1, 0, 0], [0, 1, 1, 0], [1, 0, 0, 1]],
                          [[1, 0, 1, 0], [1, 1, 0, 0], [0, 1, 0, 1]]], dtype=torch.bool)
    weight = torch.tensor([[[1.0, 0, 0, 0], [0, 3.0, 0, 0], [0, 0, 0, 5.0]],
                           [[0, 0, 2.0, 0], [4.0, 0, 0, 0], [0, 6.0, 0, 0]]])
    data = samples(torch.zeros((2, 3, 1)), torch.zeros((2, 3)), torch.tensor([[0, 1, 0], [0, 0, 0]], dtype=torch.bool),
                   torch.zeros((2, 3, 4)), torch.tensor([[0, 1, 3], [2, 0, 1]]), legal, torch.ones((2, 3, 4, 2)),
                   torch.ones((2, 3, 2)), weight, -torch.ones((2, 3)))
    s = make_compute_input_for_lossfn(TrainingLossConfig())(data)
    assert torch.equal(s.policy_mask, legal)
    assert torch.equal(s.played_action, data.played_action)
    assert torch.equal(s.beta_Q_target, data.posterior.prediction.alpha_q)
    assert torch.equal(s.beta_V_target, data.posterior.prediction.alpha_v)
    assert torch.equal(s.q_pair_weight, weight)
    assert torch.equal(s.q_supervised_pair_mask, weight > 0)
    assert torch.equal(s.value_mask, torch.tensor([[1, 1, 0], [0, 0, 0]], dtype=torch.bool))


def test_trains_root_search_targets_before_terminal_result():
    # tests/test_loss_masks.py:308-327
    data = samples(torch.zeros((3, 2, 1)), torch.zeros((3, 2)), torch.zeros((3, 2), dtype=torch.bool),
                   torch.full((3, 2, 4), 0.25), torch.zeros((3, 2), dtype=torch.int32), torch.ones((3, 2, 4), dtype=torch.bool),
                   torch.ones((3, 2, 4, 3)), torch.ones((3, 2, 3)), torch.ones((3, 2, 4)) / 4.0, -torch.ones((3, 2)))
    s = make_compute_input_for_lossfn(TrainingLossConfig(), num_outcomes=3)(data)
    assert s.policy_loss_mask.all() and s.value_loss_mask.all()
    assert not s.outcome_mask.any()


def test_preserves_search_native_target_metadata():
    # tests/test_loss_masks.py:330-382
    fields = dict(q_target_kind=torch.tensor([[[TARGET_CATEGORICAL, TARGET_DIRICHLET]]], dtype=torch.int8),
                  q_target_weight=torch.tensor([[[1.0, 0.25]]]),
                  q_target_outcome=torch.tensor([[[2, -1]]], dtype=torch.int8),
                  q_target_distance=torch.tensor([[[3, -1]]], dtype=torch.int32),
                  v_target_kind=torch.tensor([[TARGET_CATEGORICAL]], dtype=torch.int8),
                  v_target_weight=torch.tensor([[0.75]]), v_target_outcome=torch.tensor([[2]], dtype=torch.int8),
                  v_target_distance=torch.tensor([[3]], dtype=torch.int32))
    data = TrainingSamples(
        obs=torch.zeros((1, 1, 1)), reward=torch.zeros((1, 1)), terminated=torch.zeros((1, 1), dtype=torch.bool),
        discount=-torch.ones((1, 1)),
        posterior=PosteriorTargets(
            prediction=PosteriorPrediction(policy=torch.tensor([[[1.0, 0.0]]]), alpha_v=torch.ones((1, 1, 3)),
                                           alpha_q=torch.ones((1, 1, 2, 3))),
            metadata=TargetMetadata(mask=torch.ones((1, 1), dtype=torch.bool),
                                    q_supervision=QSupervision(selected=torch.ones((1, 1, 2), dtype=torch.bool),
                                                               pair_weight=torch.ones((1, 1, 2))), **fields)),
        played_action=torch.zeros((1, 1), dtype=torch.int32), legal_action_mask=torch.ones((1, 1, 2), dtype=torch.bool))
    s = make_compute_input_for_lossfn(TrainingLossConfig(), num_outcomes=3)(data)
    for name, value in fields.items():
        assert torch.equal(getattr(s, name), value), name


def _terminal_data():
    return samples(torch.zeros((1, 2, 1)), torch.tensor([[0.0, 1.0]]), torch.tensor([[False, True]]),
                   torch.ones((1, 2, 3)) / 3.0, torch.tensor([[0, 2]]), torch.ones((1, 2, 3), dtype=torch.bool),
                   torch.ones((1, 2, 3, 3)), torch.ones((1, 2, 3)), torch.zeros((1, 2, 3)),
                   torch.tensor([[-1.0, 0.0]]))


def test_can_mark_played_terminal_edge_categorical():
    # tests/test_loss_masks.py:385-407
    s = make_compute_input_for_lossfn(TrainingLossConfig(terminal_edge_targets=True), num_outcomes=3)(_terminal_data())
    assert s.q_target_kind[0, 1, 2] == TARGET_CATEGORICAL
    assert s.q_target_outcome[0, 1, 2] == 2 and s.q_target_distance[0, 1, 2] == 1
    assert s.q_pair_weight[0, 1, 2] == 1.0
    assert not (s.q_target_kind[0, 0] == TARGET_CATEGORICAL).any()
    assert not (s.q_target_kind[0, 1, :2] == TARGET_CATEGORICAL).any()


def test_can_mark_terminal_winning_parent_categorical():
    # tests/test_loss_masks.py:410-434
    s = make_compute_input_for_lossfn(TrainingLossConfig(terminal_parent_targets=True),
                                      num_outcomes=3)(_terminal_data())
    assert torch.equal(s.policy_tgt[0, 1], torch.tensor([0.0, 0.0, 1.0]))
    assert s.policy_loss_mask[0, 1] and s.value_loss_mask[0, 1]
    assert s.v_target_kind[0, 1] == TARGET_CATEGORICAL
    assert s.v_target_outcome[0, 1] == 2 and s.v_target_distance[0, 1] == 1
    assert not (s.q_target_kind == TARGET_CATEGORICAL).any()


def test_trajectory_value_targets_alternate_sign_back_from_the_result():
    # v_t = r_t + d_t v_{t+1} with d = -1 between moves and 0 at the end
    r = torch.tensor([[0.0, 0.0, 1.0, 0.0]])
    d = torch.tensor([[-1.0, -1.0, 0.0, -1.0]])
    assert torch.equal(trajectory_value_targets(r, d), torch.tensor([[1.0, -1.0, 1.0, 0.0]]))
