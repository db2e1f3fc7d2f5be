"""Writes tests/golden/block_errors_golden.npz from the reference's own code: `block_errors` (engine/quantization.py:144-169)
on the SMALL network (seed 10, weights of std 0.1 and the policy's from-projection 8 times wider, so that one block's
rounding moves the priors measurably) with its round-to-nearest int8 weights for blocks 0 and 1 (the last stays fp16).

Run in the build container, where the reference is checked out (FRY_REFERENCE, as make_golden.py reads it):

    python tests/golden/make_block_errors_golden.py

The reference's `block_errors` reads its calibration positions from a PGN through python-chess and runs on a GPU, so
this script runs its body instead. It builds the fp16 model, and the fp16 model with one block in int8, as make_golden.py
builds the reference's int8 model (`quantize_blocks`, which links the input mixes as :157-158 does). It takes their
move logits on 16 seeded boards, the softmax over each board's legal moves in fp64 (here a seeded mask of about 40
moves a board), and each block's total variation from the fp16 priors, averaged over the boards (:160-167).
"""
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))

import numpy as np
import torch

import make_golden as mg

MOVES = 1968


# wider weights than the defaults, and a sharper policy head, so that one block's rounding moves the priors measurably
STATE = {"std": 0.1, "from_scale": 8.0}


def model():
    network = mg.ref_model.ChessTransformer(**mg.SMALL).eval()
    network.load_state_dict(mg.seeded_state_dict(mg.SMALL, 10, **STATE))
    return network


def fp16_int8_model(weights: dict) -> torch.nn.Module:
    """make_golden.fp16_int8_model on the wider weights."""
    return mg.ref_int8.quantize_blocks(mg.ref_fused.FusedTransformer(model().scale_residual_stream(1 / 16).half_except_heads(torch.float16)),
                                       weights, 1 / 16)


def main() -> None:
    weights = mg.rtn_weights(model(), [0, 1])
    boards = mg.golden_boards(16, 31)
    rng = np.random.default_rng(31)
    legal = rng.random((len(boards), MOVES)) < 0.02
    legal[np.arange(len(boards)), rng.integers(0, MOVES, len(boards))] = True
    legal_t = torch.from_numpy(legal)

    def priors(int8_layers):
        with torch.no_grad():
            logits, _ = fp16_int8_model({layer: weights[layer] for layer in int8_layers})(torch.from_numpy(boards).long())
        return torch.softmax(logits.double().masked_fill(~legal_t, -torch.inf), dim=-1)

    fp16 = priors([])
    errors = [0.5 * (priors([layer]) - fp16).abs().sum(dim=-1).mean().item() for layer in (0, 1)]
    np.savez_compressed(HERE / "block_errors_golden.npz", boards=boards, legal=legal, errors=np.array(errors), fp16_priors=fp16.numpy())
    print(f"wrote {HERE / 'block_errors_golden.npz'}: errors {errors}")


if __name__ == "__main__":
    main()
