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


def test_action_layout_follows_the_reference_coordinates():
    """The reference names Hex action a by column letter a % size and row
    number a // size + 1 (scripts/checkpoint_moves.py:39-45; its vectors in
    tests/test_checkpoint_moves.py:9-21, size 5).  The restatement indexes
    cells the same way: the stone of action a lands at observation[row,
    column] of that coordinate."""
    for a, coord in [(0, "A1"), (4, "E1"), (5, "A2"), (12, "C3"), (24, "E5")]:
        column, row = ord(coord[0]) - ord("A"), int(coord[1:]) - 1
        obs = H.HexBoard(5).step(a).observation()
        # the stone belongs to the player who just moved: the opponent plane
        # of the side to move
        assert obs[row, column, 1] == 1.0 and obs[..., 1].sum() == 1.0 and obs[..., 0].sum() == 0.0


def test_initial_and_step_masks_follow_the_reference_call_site():
    """envs.py:112-131 wraps pgx.hex.Hex(size): size * size + 1 actions, the
    last (swap) never legal before a terminal state (`.at[-1].set(False)`
    on init and on every step); the empty cells are the legal moves."""
    for size in (5, 9):
        b = H.HexBoard(size)
        m = b.legal()
        assert m.shape == (size * size + 1,) and m[:-1].all() and not m[-1]
        b = b.step(size + 1)
        m = b.legal()
        assert not m[-1] and not m[size + 1] and m[:-1].sum() == size * size - 1
