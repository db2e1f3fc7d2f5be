"""The seeded legal-looking boards the golden fixtures were recorded on, regenerated without the reference.

`golden_boards(count, seed)` is the generator tests/golden/make_golden.py and make_gptq_golden.py record their
fixtures with; tests that compare against those fixtures regenerate the same boards from it.
"""
import numpy as np


def golden_boards(count: int, seed: int) -> np.ndarray:
    """Seeded legal-looking boards (each king once, 2-30 other pieces, no pawns on the back ranks, flag tokens)."""
    rng = np.random.default_rng(seed)
    boards = np.zeros((count, 70), dtype=np.uint8)
    for b in range(count):
        squares = rng.permutation(64)
        boards[b, squares[0]], boards[b, squares[1]] = 6, 12
        for square in squares[2:2 + int(rng.integers(2, 31))]:
            codes = [2, 3, 4, 5, 8, 9, 10, 11] if square < 8 or square >= 56 else [1, 2, 3, 4, 5, 7, 8, 9, 10, 11]
            boards[b, square] = rng.choice(codes)
        boards[b, 64] = 13 + rng.integers(0, 2)
        boards[b, 65:69] = 15 + rng.integers(0, 2, size=4)
        boards[b, 69] = 17 + (int(rng.integers(40, 48)) if rng.random() < 0.2 else 0)
    return boards
