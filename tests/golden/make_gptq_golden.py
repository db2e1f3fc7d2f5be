"""Writes tests/golden/gptq_golden.npz from the reference's own GPTQ (engine/quantization.py:76-99,104-140).

Run in the build container, where the reference is checked out (FRY_REFERENCE, as make_golden.py reads it):

    python tests/golden/make_gptq_golden.py

It sets up the reference's modules as make_golden.py does, then runs `compute_int8_weights` on the SMALL network (seed
10, fp64 but the heads, as engine/quantization.py:200-201 loads the model) over 64 seeded boards, recording the
(weight, hessian) that each call of the reference's `gptq` receives for block 0: the projection (K 128, one column
block) and the down matmul (padded from 320 inputs to 384 and rotated: three column blocks, 64 inputs with no
curvature). The recorded inputs are rounded to fp32 to halve the file, and the reference's `gptq` is run again on those
rounded values, so the stored outputs are exactly the reference's for the stored inputs. Block 0's raw sums from
`input_hessians` (before the down's padding and rotation) are stored too, rounded to fp32, for the layout step.
"""
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))

import numpy as np
import torch

import make_golden as mg


def main() -> None:
    real = mg.ref_quantization.gptq
    calls = []

    def recorded(weight, hessian):
        calls.append((weight.detach().clone(), hessian.detach().clone()))
        return real(weight, hessian)

    mg.ref_quantization.gptq = recorded
    boards = torch.from_numpy(mg.golden_boards(64, 21)).long()
    try:
        model = mg.reference_model(mg.SMALL, 10).half_except_heads(torch.float64)
        mg.ref_quantization.compute_int8_weights(model, boards)
        # the sums compute_int8_weights starts from (input_hessians, :103-119), block 0's
        raw = mg.ref_quantization.input_hessians(model, boards)[0]
    finally:
        mg.ref_quantization.gptq = real
    # block 0's calls, in compute_int8_weights' order: projection, gate_up, down
    out = {f"raw_{name}_hessian": raw[name].float().numpy() for name in ("projection", "gate_up", "down")}
    for name, (weight, hessian) in (("projection", calls[0]), ("down", calls[2])):
        weight32, hessian32 = weight.float(), hessian.float()
        integers, scale = real(weight32.double(), hessian32.double())
        out.update({f"{name}_weight": weight32.numpy(), f"{name}_hessian": hessian32.numpy(), f"{name}_int8": integers.numpy(),
                    f"{name}_scale": scale.numpy()})
    np.savez_compressed(HERE / "gptq_golden.npz", **out)
    print(f"wrote {HERE / 'gptq_golden.npz'}:", {k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main()
