"""Board encoding and the move table, restated without python-chess.

Follows `model/encoding.py:3-52` (token layout, vocabulary, the 1968-move
table and the promotion tables) and `model/model.py:102-120` (piece codes,
directions, knight jumps, feature row counts). Test infrastructure only.
"""
import numpy as np

NUM_SQUARES = 64
NUM_PIECE_TYPES = 6
TOKENS_PER_BOARD = 70                                   # model/encoding.py:13
NUM_PIECE_CODES = 1 + 2 * NUM_PIECE_TYPES               # :16, 0 empty, 1-6 ours, 7-12 theirs
NUM_FLAG_VALUES = 2
TURN_TOKEN_OFFSET = NUM_PIECE_CODES                     # :19
CASTLING_TOKEN_OFFSET = TURN_TOKEN_OFFSET + NUM_FLAG_VALUES
EN_PASSANT_TOKEN_OFFSET = CASTLING_TOKEN_OFFSET + NUM_FLAG_VALUES
BOARD_VOCAB_SIZE = EN_PASSANT_TOKEN_OFFSET + NUM_SQUARES  # :23, 81

# python-chess piece types, used only for the promotion order
_KNIGHT, _BISHOP, _ROOK, _QUEEN = 2, 3, 4, 5

QUEEN_STEPS = [(0, 1), (0, -1), (1, 0), (-1, 0), (1, 1), (-1, 1), (1, -1), (-1, -1)]
KNIGHT_STEPS = [(1, 2), (2, 1), (2, -1), (1, -2), (-1, -2), (-2, -1), (-2, 1), (-1, 2)]


def _destinations(square: int) -> list[int]:
    """Empty-board queen and knight destinations of a square, ascending, as
    `model/encoding.py:27-38` collects them (a SquareSet iterates ascending)."""
    f, r = square % 8, square // 8
    found = set()
    for df, dr in QUEEN_STEPS:
        nf, nr = f + df, r + dr
        while 0 <= nf < 8 and 0 <= nr < 8:
            found.add(nr * 8 + nf)
            nf, nr = nf + df, nr + dr
    for df, dr in KNIGHT_STEPS:
        if 0 <= f + df < 8 and 0 <= r + dr < 8:
            found.add((r + dr) * 8 + f + df)
    return sorted(found)


def _all_moves() -> list[tuple[int, int, int | None]]:
    """(from, to, promotion piece type or None) per move id: `model/encoding.py:25-49`."""
    moves = [(square, to, None) for square in range(NUM_SQUARES) for to in _destinations(square)]
    for from_rank, to_rank in [(6, 7), (1, 0)]:
        for from_file in range(8):
            for to_file in range(max(from_file - 1, 0), min(from_file + 2, 8)):
                for piece in (_KNIGHT, _ROOK, _BISHOP, _QUEEN):
                    moves.append((from_rank * 8 + from_file, to_rank * 8 + to_file, piece))
    return moves


ALL_MOVES = _all_moves()
NUM_MOVE_IDS = len(ALL_MOVES)                           # 1968
MOVE_FROM_SQUARES = np.array([m[0] for m in ALL_MOVES], dtype=np.int64)   # :63
MOVE_TO_SQUARES = np.array([m[1] for m in ALL_MOVES], dtype=np.int64)     # :64
PROMOTION_MOVE_IDS = np.array([i for i, m in enumerate(ALL_MOVES) if m[2] is not None], dtype=np.int64)  # :67
PROMOTION_TO_SQUARES = MOVE_TO_SQUARES[PROMOTION_MOVE_IDS]                # :68
PROMOTION_PIECES = np.array([ALL_MOVES[i][2] - _KNIGHT for i in PROMOTION_MOVE_IDS], dtype=np.int64)  # :69
ANSWER_WIDTH = NUM_MOVE_IDS + 1                         # answer rows: logits then the expected score

