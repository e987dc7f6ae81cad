"""The root target packing (scacchi_pack_targets) and the loss-input
assembly (scacchi_loss_input) kernels against the oracle restatements
(oracle.oracle.pack_targets: play_search.py:490-548 with
dirichlet_q_search.py:119-182; oracle/loss_ref.py: loss.py:164-357), bit
for bit on random inputs for every configuration, and the reference's own
loss-mask assertions (tests/test_loss_masks.py:132-434) through the
kernel."""

import numpy as np
import pytest
import torch

import tests.test_loss_input as ref_cases
from oracle import loss_ref
from oracle import oracle as O
from scacchi_b200.loss_input import LossMaskMode, PolicyTargetMode, TrainingLossConfig, make_compute_input_for_lossfn
from scacchi_b200.play import TrainingSamples
from scacchi_b200.play_search import (PosteriorPrediction, PosteriorTargets, QSupervision, TargetMetadata,
                                      pack_targets)
from scacchi_b200.types import QActionSet, QPairReduction, QSupervisionConfig

pytestmark = pytest.mark.gpu


class _Summary:
    def __init__(self, d):
        for k, v in d.items():
            setattr(self, k, torch.from_numpy(v).cuda())


def _random_summary(rng, B, A):
    visit = rng.integers(0, 4, (B, A)).astype(np.float32)
    q_out = np.where(rng.uniform(size=(B, A)) < 0.2, rng.integers(0, 2, (B, A)), -1).astype(np.int8)
    v_out = np.where(rng.uniform(size=B) < 0.3, rng.integers(0, 2, B), -1).astype(np.int8)
    return dict(visit_counts=visit, alpha=rng.uniform(0.1, 3, (B, A, 2)).astype(np.float32),
                value_alpha=rng.uniform(0.1, 3, (B, 2)).astype(np.float32), q_categorical_outcome=q_out,
                q_categorical_distance=np.where(q_out >= 0, rng.integers(0, 9, (B, A)), -1).astype(np.int32),
                v_categorical_outcome=v_out,
                v_categorical_distance=np.where(v_out >= 0, rng.integers(0, 9, B), -1).astype(np.int32))


@pytest.mark.parametrize("action_set", [0, 1])
@pytest.mark.parametrize("reduction", [0, 1])
def test_pack_targets_matches_oracle(cuda, action_set, reduction):
    rng = np.random.default_rng(7 + 2 * action_set + reduction)
    B, A = 300, 82
    s = _random_summary(rng, B, A)
    legal = rng.uniform(size=(B, A)) < 0.7
    legal[:5] = False                                   # lanes without a legal action
    policy = np.where(legal & (rng.uniform(size=(B, A)) < 0.5), rng.uniform(0, 2, (B, A)), 0).astype(np.float32)
    policy[5:9] = 0.0                                   # lanes whose search loss mask is false
    action = rng.integers(0, A, B).astype(np.int32)
    cfg = QSupervisionConfig(action_set=[QActionSet.positive_search_evidence_or_solved,
                                         QActionSet.positive_posterior_policy_or_solved][action_set],
                             reduction=[QPairReduction.mean_over_selected_state_action_pairs,
                                        QPairReduction.legacy_normalized_source_weighted_mean][reduction])
    md = pack_targets(_Summary(s), torch.from_numpy(policy).cuda(), torch.from_numpy(legal).cuda(),
                      torch.from_numpy(action).cuda(), cfg)
    torch.cuda.synchronize()
    want = O.pack_targets(s, policy, legal, action, action_set, reduction)
    got = dict(mask=md.mask, q_supervision_selected=md.q_supervision.selected,
               q_supervision_pair_weight=md.q_supervision.pair_weight,
               q_positive_evidence_action=md.q_positive_evidence_action,
               q_positive_policy_action=md.q_positive_policy_action, search_action=md.search_action,
               q_target_kind=md.q_target_kind, q_target_weight=md.q_target_weight,
               q_target_outcome=md.q_target_outcome, q_target_distance=md.q_target_distance,
               v_target_kind=md.v_target_kind, v_target_weight=md.v_target_weight,
               v_target_outcome=md.v_target_outcome, v_target_distance=md.v_target_distance)
    for k, v in got.items():
        r = np.asarray(want[k])
        assert np.array_equal(v.cpu().numpy().astype(r.dtype), r), k


def _random_frames(rng, B, T, A, metadata_mask: bool, native: bool, num_outcomes=2):
    legal = rng.uniform(size=(B, T, A)) < 0.6
    legal[0, 0] = False
    terminated = rng.uniform(size=(B, T)) < 0.15
    reward = np.where(terminated, rng.choice([-1.0, 0.0, 1.0], (B, T)), 0.0).astype(np.float32)
    discount = np.where(terminated, 0.0, -1.0).astype(np.float32)
    policy = np.where(legal, rng.uniform(0, 1, (B, T, A)), 0).astype(np.float32)
    policy[1, :3] = 0.0
    q_w = np.where(rng.uniform(size=(B, T, A)) < 0.4, rng.uniform(0, 3, (B, T, A)), 0).astype(np.float32)
    t = lambda x: torch.from_numpy(np.ascontiguousarray(x))
    fields = {}
    if native:
        fields = dict(q_target_kind=t(rng.integers(0, 3, (B, T, A)).astype(np.int8)),
                      q_target_weight=t(rng.uniform(0, 1, (B, T, A)).astype(np.float32)),
                      q_target_outcome=t(rng.integers(-1, num_outcomes, (B, T, A)).astype(np.int8)),
                      q_target_distance=t(rng.integers(-1, 9, (B, T, A)).astype(np.int32)),
                      v_target_kind=t(rng.integers(0, 3, (B, T)).astype(np.int8)),
                      v_target_weight=t(rng.uniform(0, 1, (B, T)).astype(np.float32)),
                      v_target_outcome=t(rng.integers(-1, num_outcomes, (B, T)).astype(np.int8)),
                      v_target_distance=t(rng.integers(-1, 9, (B, T)).astype(np.int32)))
    md = TargetMetadata(mask=t(rng.uniform(size=(B, T)) < 0.8) if metadata_mask else None,
                        q_supervision=QSupervision(selected=t(q_w > 0), pair_weight=t(q_w)), **fields)
    return TrainingSamples(
        obs=torch.zeros((B, T, 1)), reward=t(reward), terminated=t(terminated), discount=t(discount),
        posterior=PosteriorTargets(prediction=PosteriorPrediction(
            policy=t(policy), alpha_v=t(rng.uniform(0.5, 2, (B, T, num_outcomes)).astype(np.float32)),
            alpha_q=t(rng.uniform(0.5, 2, (B, T, A, num_outcomes)).astype(np.float32))), metadata=md),
        played_action=t(rng.integers(0, A, (B, T)).astype(np.int32)), legal_action_mask=t(legal))


def _to(samples, dev):
    def mv(x):
        if isinstance(x, torch.Tensor):
            return x.to(dev)
        if isinstance(x, tuple) and hasattr(x, "_fields"):
            return type(x)(*[mv(v) for v in x])
        return x
    return mv(samples)


CASES = [dict(), dict(loss_mask_mode=LossMaskMode.value), dict(loss_mask_mode=LossMaskMode.pgx),
         dict(policy_target_mode=PolicyTargetMode.winner_action), dict(terminal_edge_targets=True),
         dict(terminal_parent_targets=True), dict(terminal_edge_targets=True, terminal_parent_targets=True,
                                                  q_supervision=QSupervisionConfig(
                                                      reduction=QPairReduction.legacy_normalized_source_weighted_mean))]


@pytest.mark.parametrize("native", [False, True], ids=["defaults", "sidecars"])
@pytest.mark.parametrize("metadata_mask", [False, True], ids=["policy_sum", "metadata_mask"])
@pytest.mark.parametrize("case", range(len(CASES)))
def test_loss_input_matches_oracle(cuda, case, metadata_mask, native):
    rng = np.random.default_rng(100 + case * 4 + 2 * metadata_mask + native)
    frames = _random_frames(rng, 24, 17, 9, metadata_mask, native)
    cfg = TrainingLossConfig(**CASES[case])
    want = loss_ref.make_compute_input_for_lossfn(cfg)(frames)
    got = make_compute_input_for_lossfn(cfg)(_to(frames, "cuda"))
    torch.cuda.synchronize()
    for name in want._fields:
        w, g = getattr(want, name), getattr(got, name)
        if w is None:
            assert g is None, name
            continue
        w = w.cpu()
        g = g.cpu()
        assert g.shape == w.shape, name
        assert torch.equal(g.to(w.dtype), w), name


@pytest.mark.parametrize("name", [n for n in dir(ref_cases) if n.startswith("test_")
                                  and n != "test_trajectory_value_targets_alternate_sign_back_from_the_result"])
def test_reference_loss_mask_assertions_through_the_kernel(cuda, name, monkeypatch):
    """The reference's loss-mask cases, run against the kernel-backed API
    on CUDA frames."""
    def on_gpu(cfg, num_outcomes=2):
        fn = make_compute_input_for_lossfn(cfg, num_outcomes)
        return lambda frames: _to(fn(_to(frames, "cuda")), "cpu")

    monkeypatch.setattr(ref_cases, "make_compute_input_for_lossfn", on_gpu)
    getattr(ref_cases, name)()
