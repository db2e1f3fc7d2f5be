"""Seeded synthetic positions, the stand-in for the engine's MCTS leaves when benchmarking (no game data ships here).

Each board has both kings once (codes 6 and 12), 2-30 other pieces uniform over the free squares with codes uniform in
{1..5, 7..11} and no pawns on the first or last rank, then the turn, four castling flags and the en passant token, laid out
as model/encoding.py:72-92 encodes a position.
"""
import numpy as np

from .encoding import CASTLING_TOKEN_OFFSET, EN_PASSANT_TOKEN_OFFSET, TOKENS_PER_BOARD, TURN_TOKEN_OFFSET

_ANY = np.array([1, 2, 3, 4, 5, 7, 8, 9, 10, 11], dtype=np.uint8)
_NO_PAWNS = np.array([2, 3, 4, 5, 8, 9, 10, 11], dtype=np.uint8)
_BACK_RANK = np.zeros(64, dtype=bool)
_BACK_RANK[:8] = _BACK_RANK[56:] = True

# the initial position from the side to move, as encode_board gives it for chess.Board()
START_BOARD = np.array([4, 2, 3, 5, 6, 3, 2, 4] + [1] * 8 + [0] * 32 + [7] * 8 + [10, 8, 9, 11, 12, 9, 8, 10]
                       + [TURN_TOKEN_OFFSET + 1] + [CASTLING_TOKEN_OFFSET + 1] * 4 + [EN_PASSANT_TOKEN_OFFSET], dtype=np.uint8)


def random_boards(count: int, seed: int) -> np.ndarray:
    """uint8 [count, 70] boards from one seed (numpy's PCG64, the same on every machine)."""
    rng = np.random.default_rng(seed)
    boards = np.zeros((count, TOKENS_PER_BOARD), dtype=np.uint8)
    order = np.argsort(rng.random((count, 64)), axis=1)
    rows = np.arange(count)[:, None]
    boards[rows[:, 0], order[:, 0]] = 6
    boards[rows[:, 0], order[:, 1]] = 12
    others = order[:, 2:]
    pieces = np.where(_BACK_RANK[others], rng.choice(_NO_PAWNS, size=others.shape), rng.choice(_ANY, size=others.shape))
    present = np.arange(62)[None, :] < rng.integers(2, 31, size=count)[:, None]
    boards[rows, others] = np.where(present, pieces, 0)
    boards[:, 64] = TURN_TOKEN_OFFSET + rng.integers(0, 2, size=count)
    boards[:, 65:69] = CASTLING_TOKEN_OFFSET + rng.integers(0, 2, size=(count, 4))
    en_passant = np.where(rng.random(count) < 0.1, rng.integers(40, 48, size=count), 0)
    boards[:, 69] = EN_PASSANT_TOKEN_OFFSET + en_passant
    return boards
