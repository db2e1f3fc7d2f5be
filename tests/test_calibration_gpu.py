"""int8_model without weights, as the engine calls it (engine/inference.py:267-272 -> engine/quantization.py:188-207):
the checkpoint's fp64 network on the GPU sums each int8 matmul's input Hessian over the calibration positions, GPTQ
rounds every block but the last on the device, block_errors keeps the fp16_blocks worst blocks in fp16, and the weights
are cached under the checkpoint's sha256.

Pins: the fp64 network's Hessians are the reference's own (block 0 of the SMALL network over the fixture's 64 boards,
tests/golden/gptq_golden.npz); the calibrated model meets the reference's int8-vs-fp32 criterion (tests/test_int8.py:
359-373) on the reference's fp32 outputs; the choice is block_errors' own; the cache gives the same weights back
without recomputing them, and the reference's own cache file is read when no calibration is given."""
import numpy as np
import pytest
import torch

from chess_transformer_b200 import calibration, quantization
from chess_transformer_b200.build import build
from chess_transformer_b200.library import FryError
from chess_transformer_b200.network import Int8Network, geometry, int8_model
from oracle import model as om
from tests.conftest import ROOT, SMALL
from tests.golden.seeded_boards import golden_boards

pytestmark = pytest.mark.gpu

GPTQ_GOLDEN = ROOT / "tests" / "golden" / "gptq_golden.npz"


@pytest.fixture(scope="module", autouse=True)
def built():
    build()


def test_the_calibration_networks_hessians_are_the_references():
    # make_gptq_golden.py: the reference's input_hessians of its fp64 SMALL network (seed 10) over golden_boards(64, 21),
    # block 0's sums rounded to fp32
    golden = np.load(GPTQ_GOLDEN)
    model = calibration.CalibrationNetwork(om.seeded_state_dict(SMALL, 10), geometry(SMALL), "cuda")
    sums = quantization.input_hessians(model, torch.from_numpy(golden_boards(64, 21)).long().cuda())
    assert len(sums) == SMALL["num_layers"]
    for name in ("projection", "gate_up", "down"):
        found, expected = sums[0][name].cpu().numpy(), golden[f"raw_{name}_hessian"].astype(np.float64)
        assert found.shape == expected.shape and np.array_equal(found, found.T)
        assert np.allclose(found, expected, rtol=1e-6, atol=1e-6 * np.abs(expected).max()), name


def legal_masks(count: int, seed: int) -> torch.Tensor:
    rng = np.random.default_rng(seed)
    legal = np.zeros((count, 1968), dtype=bool)
    for row in legal:
        row[rng.choice(1968, size=int(rng.integers(8, 40)), replace=False)] = True
    return torch.from_numpy(legal)


def test_int8_model_calibrates_a_checkpoint_keeps_its_worst_block_fp16_and_caches_the_weights(tmp_path, monkeypatch, golden):
    monkeypatch.setenv(quantization.CACHE_VARIABLE, str(tmp_path / "cache"))
    state = om.seeded_state_dict(SMALL, 10)
    path = tmp_path / "model.pt"
    torch.save({"model_settings": SMALL, "state_dict": state}, path)  # model/checkpoint.py:22-23's format
    boards, legal = torch.from_numpy(golden_boards(64, 21)).long(), legal_masks(64, 5)
    network = int8_model(path, 1, calibration=(boards, legal))
    # the last block (FP16_LAST_LAYERS) and the block of the larger block_errors stay fp16
    all_int8 = quantization.int8_weights(path, 0, (boards, None))
    errors = quantization.block_errors(state, SMALL, all_int8, boards, legal)
    kept = quantization.fp16_choice(errors, 1)
    assert set(all_int8) == {0, 1} and len(kept) == 1
    assert [b["precision"] for b in network.blocks] == [1 if i in kept or i == 2 else 0 for i in range(3)]
    # the model is the Int8Network of those weights, and meets the reference's int8-vs-fp32 criterion
    fp32_boards = torch.from_numpy(golden["fp32_boards"]).long()
    weights = {layer: w for layer, w in all_int8.items() if layer not in kept}
    with torch.no_grad():
        rows = network(fp32_boards.cuda()).cpu()
        direct = Int8Network(state, SMALL, weights)(fp32_boards.cuda()).cpu()
    assert torch.equal(rows, direct)
    logits, values = torch.from_numpy(golden["fp32_small_logits"]), torch.from_numpy(golden["fp32_small_values"])
    distance = 0.5 * (torch.softmax(rows[:, :-1], -1) - torch.softmax(logits, -1)).abs().sum(-1)
    assert distance.max() < 0.005
    assert torch.equal(rows[:, :-1].argmax(-1), logits.argmax(-1))
    assert torch.allclose(rows[:, -1], om.expected_score(values), atol=5e-3)
    # a second start reads the cached weights: nothing is recomputed
    monkeypatch.setattr(quantization, "CalibrationNetwork", lambda *a, **k: pytest.fail("recomputed cached weights"))
    monkeypatch.setattr(quantization, "block_errors", lambda *a, **k: pytest.fail("recomputed a cached choice"))
    again = int8_model(path, 1, calibration=(boards, legal))
    with torch.no_grad():
        assert torch.equal(again(fp32_boards.cuda()).cpu(), rows)
    # without calibration: the reference's own cache file for this checkpoint, or a clear refusal
    with pytest.raises(FryError, match="calibration"):
        int8_model(path, 1)
    reference_file = quantization.cached_weights_path(path, 1)
    torch.save(weights, reference_file)
    with torch.no_grad():
        assert torch.equal(int8_model(path, 1)(fp32_boards.cuda()).cpu(), rows)
