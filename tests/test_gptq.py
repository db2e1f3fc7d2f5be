"""GPTQ (engine/quantization.py:76-99): the oracle against the reference's own outputs (tests/golden/gptq_golden.npz,
made by tests/golden/make_gptq_golden.py), and the C ABI's host refusals. No GPU."""
import ctypes

import numpy as np
import pytest

from chess_transformer_b200.build import build
from chess_transformer_b200.library import FryError, library
from oracle.gptq import gptq
from tests.conftest import ROOT

GOLDEN = ROOT / "tests" / "golden" / "gptq_golden.npz"


@pytest.mark.parametrize("name", ["projection", "down"])
def test_the_oracle_rounds_as_the_reference(name):
    # the projection: one block of 128 columns; the down matmul: 320 inputs padded to 384 and rotated, three blocks, the
    # 64 padding inputs with no curvature
    golden = np.load(GOLDEN)
    integers, scale = gptq(golden[f"{name}_weight"], golden[f"{name}_hessian"])
    assert np.array_equal(integers, golden[f"{name}_int8"])
    assert np.array_equal(scale, golden[f"{name}_scale"])
    if name == "down":
        dead = np.diagonal(golden["down_hessian"]) == 0
        assert dead.sum() == 64 and not integers[:, dead].any()


def test_gptq_is_not_rounding_to_nearest():
    # the Hessian matters: GPTQ's answer differs from round-to-nearest (its identity-Hessian case) on the same weight
    golden = np.load(GOLDEN)
    weight = golden["down_weight"].astype(np.float64)
    nearest, _ = gptq(weight, np.eye(weight.shape[1]))
    scale = np.abs(weight).max(axis=1, keepdims=True) / 127
    assert np.array_equal(nearest, np.clip(np.rint(weight / scale), -127, 127).astype(np.int8))
    assert (golden["down_int8"] != nearest).mean() > 0.05


def test_gptq_is_refused_on_the_host_before_any_cuda_call():
    build()
    lib = library()
    buffer = ctypes.c_void_p(16)
    with pytest.raises(FryError, match="0 < K <= 4096"):
        lib.fry_gptq(buffer, buffer, 8, 5000, buffer, buffer, buffer, 1 << 40, None)
    with pytest.raises(FryError, match="0 < N"):
        lib.fry_gptq(buffer, buffer, 0, 128, buffer, buffer, buffer, 1 << 40, None)
    with pytest.raises(FryError, match="workspace is smaller"):
        lib.fry_gptq(buffer, buffer, 8, 128, buffer, buffer, buffer, 16, None)
    with pytest.raises(FryError, match="needs its weight"):
        lib.fry_gptq(None, buffer, 8, 128, buffer, buffer, buffer, 1 << 40, None)
    assert lib.fry_gptq_workspace_bytes(0, 128) == 0 and lib.fry_gptq_workspace_bytes(768, 1024) >= (2 * 1024 * 1024 + 768 * 1024) * 8


def test_the_layout_gptq_takes_is_the_references():
    # engine/quantization.py:129-139: from block 0's raw sums (input_hessians, :103-119) to the (weight, hessian) pairs the
    # reference's gptq received: the projection's rows Q|K|V|template mix with its sums, the down's padded and rotated pair
    import torch
    from chess_transformer_b200.quantization import gptq_inputs
    from oracle import model as om
    from tests.conftest import SMALL
    golden = np.load(GOLDEN)
    sums = {name: torch.from_numpy(golden[f"raw_{name}_hessian"]).double() for name in ("projection", "gate_up", "down")}
    pairs = gptq_inputs(om.seeded_state_dict(SMALL, 10), 0, sums)
    assert torch.equal(pairs["projection"][0].float(), torch.from_numpy(golden["projection_weight"]))
    assert torch.equal(pairs["projection"][1].float(), torch.from_numpy(golden["projection_hessian"]))
    assert torch.allclose(pairs["down"][0].float(), torch.from_numpy(golden["down_weight"]), rtol=1e-6, atol=0)
    recorded = torch.from_numpy(golden["down_hessian"]).double()
    # the recorded pair was rotated from the fp64 sums; these are the sums rounded to fp32 first
    assert torch.allclose(pairs["down"][1], recorded, rtol=1e-5, atol=1e-6 * recorded.abs().max().item())
    assert pairs["gate_up"][0].shape == (2 * SMALL["mlp_hidden"], SMALL["d_model"])


def test_the_fp16_choice_keeps_the_blocks_of_the_largest_errors():
    # engine/quantization.py:196-198
    from chess_transformer_b200.quantization import fp16_choice
    errors = {0: 0.01, 1: 0.04, 2: 0.02, 3: 0.03}
    assert fp16_choice(errors, 1) == [1] and fp16_choice(errors, 2) == [1, 3] and fp16_choice(errors, 0) == []
