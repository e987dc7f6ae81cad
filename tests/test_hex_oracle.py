"""The Hex restatement on known positions (CPU)."""

import numpy as np

from oracle import hex_ref as H


def play(size, moves, black_player=0):
    b = H.HexBoard(size, black_player)
    for m in moves:
        b = b.step(m)
    return b


def cell(size, r, c):
    return r * size + c


def test_black_column_wins_top_to_bottom():
    s = 9
    moves = []
    for r in range(s):
        moves.append(cell(s, r, 4))          # black down column 4
        if r < s - 1:
            moves.append(cell(s, r, 0))      # white along column 0 (no left-right link)
    b = play(s, moves)
    assert b.terminated and b.winner == 0 and b.color == 1
    assert b.rewards().tolist() == [1.0, -1.0]
    assert b.legal().all()  # every action reads legal at a terminal state


def test_white_row_wins_left_to_right_and_rewards_follow_player_order():
    s = 5
    moves = []
    for c in range(s):
        moves.append(cell(s, 0 if c % 2 else 4, c) if c < s - 1 else cell(s, 1, 4))  # black scattered
        moves.append(cell(s, 2, c))          # white along row 2
    b = H.HexBoard(s, black_player=1)
    for m in moves:
        if b.terminated:
            break
        b = b.step(m)
    assert b.terminated and b.winner == 1
    # black is player 1, so white (the winner) is player 0
    assert b.rewards().tolist() == [1.0, -1.0]


def test_anti_diagonal_connects_but_main_diagonal_does_not():
    s = 5
    anti = [cell(s, r, s - 1 - r) for r in range(s)]      # (r+1, c-1) neighbours
    white = [cell(s, 0, 0), cell(s, 1, 0), cell(s, 2, 0), cell(s, 3, 0)]
    b = play(s, [m for pair in zip(anti, white + [None]) for m in pair if m is not None])
    assert b.terminated and b.winner == 0
    diag = [cell(s, r, r) for r in range(s)]              # (r+1, c+1) are not neighbours
    white2 = [cell(s, 0, 4), cell(s, 1, 4), cell(s, 2, 4), cell(s, 3, 4)]
    b2 = play(s, [m for pair in zip(diag, white2 + [None]) for m in pair if m is not None])
    assert not b2.terminated


def test_record_round_trip_and_observation():
    s = 9
    b = play(s, [0, 80, 40], black_player=1)
    rec = b.record()
    assert rec.shape == (48,)
    c = H.HexBoard.from_record(rec)
    assert np.array_equal(c.cells, b.cells) and c.color == 1 and c.black_player == 1 and c.moves == 3
    obs = b.observation()  # white to move
    assert obs[8, 8, 0] == 1 and obs[0, 0, 1] == 1 and obs[4, 4, 1] == 1
    assert (obs[..., 2] == 1).all() and (obs[..., 3] == 0).all()
    assert play(s, [5]).observation()[..., 3].all()  # second move
    legal = b.legal()
    assert not legal[-1] and not legal[0] and legal[1] and legal.sum() == 78
    assert b.current_player() == 0  # white is player 0 when black is player 1


def test_step_outputs_terminal_outcome_is_a_loss_for_the_child():
    s = 3
    # black: (0,1) (1,1) then (2,1) connects; white plays column 0
    rec = play(s, [1, 0, 4, 3]).record()
    out = H.step_outputs(rec, 7)
    assert out["terminated"] and out["terminal"] == 0 and out["to_play"] == 1
    # an occupied cell leaves the state unchanged
    same = H.step_outputs(rec, 1)
    assert np.array_equal(same["record"], rec) and same["terminal"] == -1


def test_random_roots_are_reproducible_and_in_range():
    from oracle import oracle as O

    key = O.PRNGKey(3)
    boards = [H.random_root(9, key, lane, 0, 20) for lane in range(64)]
    assert all(0 <= b.moves <= 20 for b in boards)
    assert len({b.moves for b in boards}) > 5
    again = H.random_root(9, key, 17, 0, 20)
    assert np.array_equal(again.record(), boards[17].record())
