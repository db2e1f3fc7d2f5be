"""block_errors (engine/quantization.py:144-169), the ranking that picks the blocks kept in fp16, against the reference's
own values (tests/golden/block_errors_golden.npz, made by tests/golden/make_block_errors_golden.py)."""
import numpy as np
import pytest
import torch

from chess_transformer_b200.build import build
from chess_transformer_b200.network import Int8Network, quantize
from chess_transformer_b200.quantization import block_errors, fp16_choice
from oracle import model as om
from tests.conftest import ROOT, SMALL

pytestmark = pytest.mark.gpu

GOLDEN = ROOT / "tests" / "golden" / "block_errors_golden.npz"
STATE = {"std": 0.1, "from_scale": 8.0}  # the fixture's weights (make_block_errors_golden.py)


@pytest.fixture(scope="module", autouse=True)
def built():
    build()


def test_block_errors_are_the_references():
    # The fp16 blocks here sum their products in fp32 where the reference's sum in fp16 (model/fused_blocks.py:291), and
    # each network's priors sit within that of the reference's. So each block's error is the reference's to within 20%,
    # and the ranking, which is all the choice reads, is the same.
    golden = np.load(GOLDEN)
    state = om.seeded_state_dict(SMALL, 10, **STATE)
    weights = quantize(state, SMALL, [0, 1])
    boards, legal = torch.from_numpy(golden["boards"]).long(), torch.from_numpy(golden["legal"])
    errors = block_errors(state, SMALL, weights, boards, legal)
    expected = golden["errors"]
    assert set(errors) == {0, 1}
    assert np.allclose([errors[0], errors[1]], expected, rtol=0.2, atol=0)
    assert fp16_choice(errors, 1) == [int(np.argmax(expected))]
    with torch.no_grad():
        logits = Int8Network(state, SMALL, {})(boards.cuda())[:, :-1]
    fp16 = torch.softmax(logits.double().masked_fill(~legal.cuda(), -torch.inf), dim=-1).cpu().numpy()
    assert 0.5 * np.abs(fp16 - golden["fp16_priors"]).sum(-1).mean() <= 0.2 * expected.min()
