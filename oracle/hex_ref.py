"""Hex environment restated on the CPU (numpy + Python loops).

TEST INFRASTRUCTURE ONLY: the checker for the CUDA Hex kernels.

The reference builds its Hex environment on pgx 2.6.0 (`scacchi/envs.py:98-125`):
`pgx.hex.Hex(size)` with a random player order drawn by `bernoulli(key)` at
init, the swap action always masked, and rewards indexed by player order.
pgx itself is not installed here, so this file restates the rules of Hex:

* cells are indexed r * size + c; a cell's neighbours are (r-1, c),
  (r-1, c+1), (r, c-1), (r, c+1), (r+1, c-1), (r+1, c);
* black (colour 0) moves first and connects row 0 to row size-1; white
  (colour 1) connects column 0 to column size-1; the mover of a connecting
  stone wins (+1, the other player -1);
* after a move the colour to move flips, terminal or not;
* the legal mask is the empty cells plus a never-legal swap action; at a
  terminal state every action reads legal (pgx's convention at terminals);
* the observation for the player to move is four planes: own stones,
  opponent stones, own colour (all 0 black / all 1 white), and 1 on the
  second move of the game (when pgx's swap rule would apply).

The state record (48 bytes, shared bit for bit with the kernels):
  [0:16)  black stones, bit r*size+c of two little-endian uint64 words
  [16:32) white stones
  [32] colour to move, [33] player id playing black, [34] terminated,
  [35] winning colour (int8, -1 none), [36] size, [37] stones placed,
  [38:48) zero.
"""

from __future__ import annotations

import numpy as np

RECORD_BYTES = 48
NEIGHBOURS = ((-1, 0), (-1, 1), (0, -1), (0, 1), (1, -1), (1, 0))


class HexBoard:
    """One lane's state."""

    def __init__(self, size: int, black_player: int = 0):
        self.size = size
        self.cells = np.zeros(size * size, np.int8)  # 0 empty, 1 black, 2 white
        self.color = 0
        self.black_player = black_player
        self.terminated = False
        self.winner = -1
        self.moves = 0

    # ---- serialisation
    def record(self) -> np.ndarray:
        rec = np.zeros(RECORD_BYTES, np.uint8)
        for colour, off in ((1, 0), (2, 16)):
            bits = 0
            for i in np.nonzero(self.cells == colour)[0]:
                bits |= 1 << int(i)
            rec[off:off + 16] = np.frombuffer(bits.to_bytes(16, "little"), np.uint8)
        rec[32] = self.color
        rec[33] = self.black_player
        rec[34] = int(self.terminated)
        rec[35] = np.uint8(self.winner & 0xFF)
        rec[36] = self.size
        rec[37] = self.moves
        return rec

    @classmethod
    def from_record(cls, rec: np.ndarray) -> "HexBoard":
        rec = np.asarray(rec, np.uint8)
        b = cls(int(rec[36]), int(rec[33]))
        black = int.from_bytes(rec[0:16].tobytes(), "little")
        white = int.from_bytes(rec[16:32].tobytes(), "little")
        for i in range(b.size * b.size):
            if black >> i & 1:
                b.cells[i] = 1
            elif white >> i & 1:
                b.cells[i] = 2
        b.color = int(rec[32])
        b.terminated = bool(rec[34])
        b.winner = int(np.int8(rec[35].astype(np.int8)))
        b.moves = int(rec[37])
        return b

    # ---- rules
    def current_player(self) -> int:
        return self.black_player if self.color == 0 else 1 - self.black_player

    def connected(self, colour: int) -> bool:
        """Breadth-first search from the colour's first edge to its second."""
        s, mark = self.size, colour + 1
        start = [(0, c) for c in range(s)] if colour == 0 else [(r, 0) for r in range(s)]
        seen = set()
        frontier = [(r, c) for r, c in start if self.cells[r * s + c] == mark]
        seen.update(frontier)
        while frontier:
            r, c = frontier.pop()
            if (colour == 0 and r == s - 1) or (colour == 1 and c == s - 1):
                return True
            for dr, dc in NEIGHBOURS:
                rr, cc = r + dr, c + dc
                if 0 <= rr < s and 0 <= cc < s and (rr, cc) not in seen and self.cells[rr * s + cc] == mark:
                    seen.add((rr, cc))
                    frontier.append((rr, cc))
        return False

    def step(self, action: int) -> "HexBoard":
        """A legal cell action on a non-terminal state."""
        assert not self.terminated and 0 <= action < self.size * self.size and self.cells[action] == 0
        nxt = HexBoard(self.size, self.black_player)
        nxt.cells = self.cells.copy()
        nxt.cells[action] = self.color + 1
        nxt.moves = self.moves + 1
        if nxt.connected(self.color):
            nxt.terminated = True
            nxt.winner = self.color
        nxt.color = 1 - self.color
        return nxt

    def legal(self) -> np.ndarray:
        A = self.size * self.size + 1
        if self.terminated:
            return np.ones(A, bool)
        m = np.zeros(A, bool)
        m[:-1] = self.cells == 0
        return m

    def rewards(self) -> np.ndarray:
        r = np.zeros(2, np.float32)
        if self.terminated:
            win_player = self.black_player if self.winner == 0 else 1 - self.black_player
            r[win_player] = 1.0
            r[1 - win_player] = -1.0
        return r

    def observation(self) -> np.ndarray:
        s = self.size
        own, opp = self.color + 1, 2 - self.color
        obs = np.zeros((s, s, 4), np.float32)
        obs[..., 0] = (self.cells == own).reshape(s, s)
        obs[..., 1] = (self.cells == opp).reshape(s, s)
        obs[..., 2] = self.color
        obs[..., 3] = 1.0 if self.moves == 1 else 0.0
        return obs


def step_outputs(rec: np.ndarray, action: int) -> dict:
    """What the recurrent function of the reference derives from one step
    (dirichlet_q_search.py:43-76): the child record, its observation and
    legal mask, and the terminal outcome aligned to the child's player."""
    parent = HexBoard.from_record(rec)
    a = int(action)
    legal = not parent.terminated and 0 <= a < parent.size ** 2 and parent.cells[a] == 0
    # an illegal action or a terminal parent returns the state unchanged (the
    # search steps lanes with nothing to expand with action 0)
    child = parent.step(a) if legal else HexBoard.from_record(rec)
    parent_player = parent.current_player()
    reward = child.rewards()[parent_player]
    outcome = (int(np.round(reward)) + 1) // 2
    to_play = child.current_player()
    aligned = outcome if to_play == parent_player else 1 - outcome
    return dict(record=child.record(), observation=child.observation(), invalid=~child.legal(),
                terminal=aligned if child.terminated else -1, to_play=to_play, rewards=child.rewards(),
                terminated=child.terminated)


# ---- seeded roots (the full-step workload's root sampler) -----------------

def random_root(size: int, key, lane: int, min_moves: int, max_moves: int) -> HexBoard:
    """Lane `lane`'s root: player order from bernoulli(fold_in(k, 0)), then
    min_moves + bits(fold_in(k, 1)) % (max_moves - min_moves + 1) uniform
    random legal moves (move j picks the bits(fold_in(k, 2 + j)) % n-th
    empty cell in index order), stopping early at a terminal state; k =
    fold_in(key, lane)."""
    from oracle import oracle as O

    k = O.fold_in(key, lane)
    black_player = 1 if O.uniform(O.fold_in(k, 0), 1)[0] < 0.5 else 0
    board = HexBoard(size, black_player)
    n = min_moves + int(O.random_bits(O.fold_in(k, 1), 1)[0]) % (max_moves - min_moves + 1)
    for j in range(n):
        if board.terminated:
            break
        empty = np.nonzero(board.cells == 0)[0]
        pick = int(O.random_bits(O.fold_in(k, 2 + j), 1)[0]) % len(empty)
        board = board.step(int(empty[pick]))
    return board


def init_state(size: int, key) -> HexBoard:
    """envs.py:103-112 for one lane: player_order = [[0,1],[1,0]][bernoulli(key)]."""
    from oracle import oracle as O

    return HexBoard(size, 1 if O.uniform(key, 1)[0] < 0.5 else 0)
