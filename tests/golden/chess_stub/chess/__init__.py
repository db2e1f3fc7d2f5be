"""A minimal stand-in for python-chess (1.11.2), enough for the reference's
`model/encoding.py` to import: empty-board queen and knight attack sets, moves
and the constants the move table is built from.

python-chess is not installed in the build container. This stub exists only so
`tests/golden/make_golden.py` can import the reference's model code and record
its outputs as fixtures. Nothing in the product imports it.
"""

Color = bool
Square = int
PieceType = int
WHITE, BLACK = True, False
PAWN, KNIGHT, BISHOP, ROOK, QUEEN, KING = 1, 2, 3, 4, 5, 6
PIECE_TYPES = [PAWN, KNIGHT, BISHOP, ROOK, QUEEN, KING]
SQUARES = list(range(64))


def square(file_index, rank_index):
    return rank_index * 8 + file_index


def square_file(sq):
    return sq & 7


def square_rank(sq):
    return sq >> 3


def square_mirror(sq):
    return sq ^ 0x38


class Piece:
    def __init__(self, piece_type, color):
        self.piece_type, self.color = piece_type, color


class Move:
    def __init__(self, from_square, to_square, promotion=None):
        self.from_square, self.to_square, self.promotion = from_square, to_square, promotion

    def _key(self):
        return (self.from_square, self.to_square, self.promotion)

    def __eq__(self, other):
        return isinstance(other, Move) and self._key() == other._key()

    def __hash__(self):
        return hash(self._key())

    def __repr__(self):
        return f"Move({self.from_square}, {self.to_square}, {self.promotion})"


_QUEEN_STEPS = [(0, 1), (0, -1), (1, 0), (-1, 0), (1, 1), (-1, 1), (1, -1), (-1, -1)]
_KNIGHT_STEPS = [(1, 2), (2, 1), (2, -1), (1, -2), (-1, -2), (-2, -1), (-2, 1), (-1, 2)]


def _on_board(file_index, rank_index):
    return 0 <= file_index < 8 and 0 <= rank_index < 8


class Board:
    """Only what empty-board attack generation needs: pieces never block here
    because the reference builds its move table one piece at a time."""

    def __init__(self):
        self._pieces = {}

    @classmethod
    def empty(cls):
        return cls()

    def set_piece_at(self, sq, piece):
        self._pieces[sq] = piece

    def remove_piece_at(self, sq):
        self._pieces.pop(sq, None)

    def attacks(self, sq):
        piece = self._pieces[sq]
        f, r = square_file(sq), square_rank(sq)
        found = set()
        if piece.piece_type == QUEEN:
            for df, dr in _QUEEN_STEPS:
                nf, nr = f + df, r + dr
                while _on_board(nf, nr):
                    target = square(nf, nr)
                    found.add(target)
                    if target in self._pieces:
                        break
                    nf, nr = nf + df, nr + dr
        elif piece.piece_type == KNIGHT:
            for df, dr in _KNIGHT_STEPS:
                if _on_board(f + df, r + dr):
                    found.add(square(f + df, r + dr))
        else:
            raise NotImplementedError("the stub attacks with queens and knights only")
        return SquareSet(found)


class SquareSet:
    """Iterates squares in ascending order, as python-chess's SquareSet does."""

    def __init__(self, squares):
        self._squares = set(squares)

    def union(self, other):
        return SquareSet(self._squares | other._squares)

    def __iter__(self):
        return iter(sorted(self._squares))

    def __len__(self):
        return len(self._squares)
