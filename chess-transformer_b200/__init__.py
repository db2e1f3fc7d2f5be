"""fry-b200: a B200-native (sm_100a) int8 inference engine for the network of Fry (GilliamWong/chess-transformer).

The drop-in for the reference's `engine.inference.int8_model` (engine/inference.py:267-272) is `int8_model`, which
returns an `Int8Network`: `forward(boards: LongTensor[B, 70] on cuda) -> Tensor[B, 1969] fp32`, the answer rows the
search consumes. The kernels are in `libfry_b200.so` (built from csrc/ by build.py); `ops` mirrors the reference's torch
custom ops one by one; `runtime.NativeBatches` replays the forward as CUDA graphs from pinned host buffers through the
library's C++ lanes.
"""
from .encoding import ANSWER_WIDTH, NUM_MOVE_IDS, TOKENS_PER_BOARD
from .library import FryError, library

__all__ = ["ANSWER_WIDTH", "NUM_MOVE_IDS", "TOKENS_PER_BOARD", "FryError", "library"]
