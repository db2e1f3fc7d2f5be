"""The whole int8 forward (Int8Network -> fry_forward) against the oracle, the reference's own int8 model outputs and the
fp32 model, on the reference's small checkpoints and on Fry's full 28-block geometry; then the properties that hold at
any size (a board's answer does not depend on its batch), CUDA-graph lanes, and host-visible fault reporting."""
import numpy as np
import pytest
import torch

from chess_transformer_b200.boards import random_boards
from chess_transformer_b200.build import build
from chess_transformer_b200.library import library
from chess_transformer_b200.network import FRY_SETTINGS, Int8Network
from chess_transformer_b200.runtime import GraphedBatches, small_graph_sizes
from oracle import int8 as oi, model as om
from tests.conftest import SMALL, TINY

pytestmark = pytest.mark.gpu

# the north star's bar: max |logit error| <= 1e-2, |expected score error| <= 1e-3
LOGIT_TOLERANCE, SCORE_TOLERANCE = 1e-2, 1e-3


@pytest.fixture(scope="module", autouse=True)
def built():
    build()


def network_and_oracle(settings, seed, **weights_kwargs):
    state = om.seeded_state_dict(settings, seed, **weights_kwargs)
    weights = oi.int8_weights(state, settings)
    return Int8Network(state, settings, weights), oi.prepare(state, settings, weights)


@pytest.mark.parametrize("name, settings, seed", [("small", SMALL, 10), ("tiny", TINY, 11)])
def test_the_network_is_the_references_int8_model(golden, name, settings, seed):
    network, prepared = network_and_oracle(settings, seed)
    boards = torch.from_numpy(golden["fp32_boards"][:4]).long()
    with torch.no_grad():
        rows = network(boards.cuda()).cpu()
    logits, values = torch.from_numpy(golden[f"int8_{name}_logits"]), torch.from_numpy(golden[f"int8_{name}_values"])
    assert (rows[:, :-1] - logits).abs().max() <= LOGIT_TOLERANCE
    assert (rows[:, -1] - om.expected_score(values)).abs().max() <= SCORE_TOLERANCE
    assert torch.equal(rows[:, :-1].argmax(-1), logits.argmax(-1))
    expected = oi.int8_forward(prepared, boards)
    assert (rows - expected).abs().max() <= LOGIT_TOLERANCE


def test_the_network_computes_what_the_fp32_model_does(golden):
    # tests/test_int8.py:359-373: policy total variation < 0.005, the same best move, expected score within 5e-3
    network, _ = network_and_oracle(SMALL, 10)
    boards = torch.from_numpy(golden["fp32_boards"]).long()
    with torch.no_grad():
        rows = network(boards.cuda()).cpu()
    logits, values = torch.from_numpy(golden["fp32_small_logits"]), torch.from_numpy(golden["fp32_small_values"])
    distance = 0.5 * (torch.softmax(rows[:, :-1], -1) - torch.softmax(logits, -1)).abs().sum(-1)
    assert distance.max() < 0.005
    assert torch.equal(rows[:, :-1].argmax(-1), logits.argmax(-1))
    assert torch.allclose(rows[:, -1], om.expected_score(values), atol=5e-3)


@pytest.fixture(scope="module")
def fry():
    return network_and_oracle(FRY_SETTINGS, 1, std=0.02, template_std=0.02, table_std=0.02)


def test_the_28_block_fry_network_is_the_oracle(fry):
    network, prepared = fry
    boards = torch.from_numpy(random_boards(4, 11)).long()
    with torch.no_grad():
        rows = network(boards.cuda()).cpu()
    expected = oi.int8_forward(prepared, boards)
    assert rows.shape == (4, 1969) and torch.isfinite(rows).all()
    assert (rows[:, :-1] - expected[:, :-1]).abs().max() <= LOGIT_TOLERANCE
    assert (rows[:, -1] - expected[:, -1]).abs().max() <= SCORE_TOLERANCE


@pytest.mark.parametrize("batch", [64, 256])
def test_a_boards_answer_does_not_depend_on_its_batch(fry, batch):
    network, _ = fry
    boards = torch.from_numpy(random_boards(batch, batch)).long().cuda()
    with torch.no_grad():
        whole = network(boards)
        picked = [0, batch // 2, batch - 1]
        alone = network(boards[picked])
    assert torch.equal(whole[picked], alone)


def test_graph_lanes_give_the_eager_bits(fry):
    network, _ = fry
    boards = random_boards(24, 5)
    with torch.no_grad():
        eager = network(torch.from_numpy(boards).long().cuda()).cpu().numpy()
    batches = GraphedBatches(network, small_graph_sizes(24), in_flight=2)
    first = batches.launch(boards[:10])
    second = batches.launch(boards)
    assert np.array_equal(batches.collect(second), eager)
    assert np.array_equal(batches.collect(first), eager[:10])
    for _ in range(20):
        assert np.array_equal(batches.collect(batches.launch(boards[:17])), eager[:17])


def test_a_token_outside_the_vocabulary_is_reported_not_faulted(fry):
    network, _ = fry
    lib = library()
    lib.device_status(clear=True)
    boards = torch.from_numpy(random_boards(2, 0)).long()
    boards[1, 3] = 99
    with torch.no_grad():
        rows = network(boards.cuda())
    torch.cuda.synchronize()
    code, where = lib.device_status(clear=True)
    assert (code, where) == (2, 1) and torch.isfinite(rows).all()
    assert lib.device_status() == (0, 0)
