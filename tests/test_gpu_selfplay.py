"""Self-play frames (scacchi/play.py:93-175) on Hex 5x5 with a deterministic
evaluator: every frame is replayed on the Hex restatement."""

import numpy as np
import pytest
import torch

from oracle import hex_ref as H

pytestmark = pytest.mark.gpu


def test_play_training_frames_replay_on_the_restatement(cuda):
    from oracle import oracle as O
    from scacchi_b200 import random as R
    from scacchi_b200.hex import HexGame
    from scacchi_b200.play import play_training
    from scacchi_b200.play_search import EvaluatorOutput, make_search_player
    from scacchi_b200.types import (ActionCommitmentConfig, ActionCommitmentType, DirichletThompsonSearchConfig,
                                    MonteCarloPosteriorUpdateConfig, PosteriorUpdateConfig, SearchConfig,
                                    SearchKind)
    import test_gpu_hex as TH

    size, B, T, N = 5, 8, 30, 8
    game = HexGame(size)

    def model(obs):
        lg, av, aq = TH.toy_evaluator_np(obs.cpu().numpy())
        return EvaluatorOutput(logits=torch.from_numpy(lg).cuda(), alpha_v=torch.from_numpy(av).cuda(),
                               alpha_q=torch.from_numpy(aq).cuda())

    cfg = SearchConfig(kind=SearchKind.dirichlet_thompson, dirichlet_thompson=DirichletThompsonSearchConfig(
        num_simulations=N, posterior_update=PosteriorUpdateConfig(
            monte_carlo=MonteCarloPosteriorUpdateConfig(kappa=1.0, policy_samples=4))))
    player = make_search_player(game, model, cfg, ActionCommitmentConfig(kind=ActionCommitmentType.posterior_sample))
    key = R.PRNGKey(3)
    data = play_training(game, player, key, batch_size=B, max_num_steps=T)
    torch.cuda.synchronize()
    obs = data.obs.cpu().numpy()
    acts = data.played_action.cpu().numpy()
    legal = data.legal_action_mask.cpu().numpy()
    reward = data.reward.cpu().numpy()
    term = data.terminated.cpu().numpy()
    disc = data.discount.cpu().numpy()
    assert obs.shape == (B, T, size, size, 4) and data.posterior.prediction.policy.shape == (B, T, size * size + 1)
    # replay: per-lane init keys, the rollout keys' reset keys, played actions
    rollout, init_key = O.split(np.asarray(key, np.uint32))
    boards = [H.init_state(size, k) for k in O.split(init_key, B)]
    step_keys = O.split(rollout, T)
    games = 0
    for t in range(T):
        _, reset_key = O.split(step_keys[t])
        reset_keys = O.split(reset_key, B)
        for b in range(B):
            bd = boards[b]
            np.testing.assert_array_equal(obs[b, t], bd.observation())
            np.testing.assert_array_equal(legal[b, t], bd.legal())
            assert legal[b, t, acts[b, t]]
            actor = bd.current_player()
            nxt = bd.step(int(acts[b, t]))
            assert term[b, t] == nxt.terminated
            assert reward[b, t] == nxt.rewards()[actor]
            assert disc[b, t] == (0.0 if nxt.terminated else -1.0)
            if nxt.terminated:
                games += 1
                assert reward[b, t] == 1.0  # the mover of a connecting stone wins
                nxt = H.init_state(size, O.split(reset_keys[b])[1])
            boards[b] = nxt
    assert games >= B  # 30 frames of 5x5 finish at least one game per lane
    # loss input on the device frames (loss.py:164-357): value targets of a
    # finished game alternate +-1 back from its winning move, and the value
    # mask covers exactly the frames whose game ends inside the window
    from scacchi_b200.loss_input import TrainingLossConfig, make_compute_input_for_lossfn

    s = make_compute_input_for_lossfn(TrainingLossConfig(terminal_parent_targets=True))(data)
    vt = s.value_tgt.cpu().numpy()
    vm = s.value_mask.cpu().numpy()
    for b in range(B):
        last = np.nonzero(term[b])[0]
        assert np.array_equal(vm[b], np.arange(T) <= last[-1])
        sign = 1.0
        for t in range(last[-1], -1, -1):
            if term[b, t]:
                sign = 1.0
            assert vt[b, t] == sign
            sign = -sign
    assert s.value_tgt.is_cuda and s.policy_tgt.shape == (B, T, size * size + 1)
    win = term & (reward > 0)
    assert np.array_equal(s.policy_tgt.cpu().numpy()[win].argmax(-1), acts[win])
    assert (s.v_target_outcome.cpu().numpy()[win] == 1).all()
