"""The whole int8 forward (Int8Network -> fry_forward) against the oracle, the reference's own int8 model outputs and the
fp32 model, on the reference's small checkpoints and on Fry's full 28-block geometry; then the properties that hold at
any size (a board's answer does not depend on its batch), CUDA-graph lanes, and host-visible fault reporting."""
import numpy as np
import pytest
import torch

from chess_transformer_b200.boards import random_boards
from chess_transformer_b200.build import build
from chess_transformer_b200.encoding import ANSWER_WIDTH, LEAN_COLUMNS, LEAN_ROW, TOKENS_PER_BOARD
from chess_transformer_b200.library import library
from chess_transformer_b200.network import FRY_SETTINGS, Int8Network
from chess_transformer_b200.runtime import NativeBatches, lane_sizes
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


def test_the_references_layout_with_an_fp16_last_block_is_its_int8_model(golden):
    # engine/inference.py:265-272: every block int8 but the last, which runs as the fp16 FusedBlock
    # (model/fused_blocks.py:325-354); the reference's fp16 linears accumulate in fp16, these in fp32
    state = om.seeded_state_dict(SMALL, 10)
    layers = SMALL["num_layers"]
    weights = {layer: w for layer, w in oi.int8_weights(state, SMALL).items() if layer < layers - 1}
    network = Int8Network(state, SMALL, weights)
    assert [b["precision"] for b in network.blocks] == [0] * (layers - 1) + [1]
    boards = torch.from_numpy(golden["fp32_boards"][:4]).long()
    with torch.no_grad():
        rows = network(boards.cuda()).cpu()
    logits = torch.from_numpy(golden["int8_small_layout_logits"])
    values = torch.from_numpy(golden["int8_small_layout_values"])
    assert (rows[:, :-1] - logits).abs().max() <= LOGIT_TOLERANCE
    assert (rows[:, -1] - om.expected_score(values)).abs().max() <= SCORE_TOLERANCE


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
def test_the_measured_batches_are_the_oracle_and_a_boards_answer_does_not_depend_on_its_batch(fry, batch):
    # the bench's own configurations (64 boards: the engine's default batch; 256: the metric's), the whole batch on the
    # GPU, six of its rows against the oracle's forward of those boards, and the same rows run alone
    network, prepared = fry
    boards = torch.from_numpy(random_boards(batch, batch)).long()
    with torch.no_grad():
        whole = network(boards.cuda()).cpu()
        picked = [0, 1, batch // 3, batch // 2, 2 * batch // 3, batch - 1]
        alone = network(boards[picked].cuda()).cpu()
    expected = oi.int8_forward(prepared, boards[picked])
    assert torch.isfinite(whole).all()
    assert (whole[picked, :-1] - expected[:, :-1]).abs().max() <= LOGIT_TOLERANCE
    assert (whole[picked, -1] - expected[:, -1]).abs().max() <= SCORE_TOLERANCE
    assert torch.equal(whole[picked], alone)


class Recorded:
    """The forward as a caller's runtime records it (the reference's contract, engine/inference.py:117-125): on a side
    stream, after an eager warm-up there, one CUDA graph per batch size sharing one private memory pool, each reading a
    fixed device input buffer and leaving its answers in a fixed output. replay(n) runs the size-n graph on the stream."""

    def __init__(self, answer, inputs: torch.Tensor, sizes: list[int]):
        self.stream, self.inputs, self.graphs, self.outputs = torch.cuda.Stream(), inputs, {}, {}
        self.stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(self.stream), torch.no_grad():
            for size in sizes:
                answer(inputs[:size])
        pool = torch.cuda.graph_pool_handle()
        for size in sorted(sizes, reverse=True):
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, pool=pool, stream=self.stream), torch.no_grad():
                self.outputs[size] = answer(inputs[:size])
            self.graphs[size] = graph
        self.stream.synchronize()

    def replay(self, host_inputs: np.ndarray) -> np.ndarray:
        count = len(host_inputs)
        size = min(s for s in self.graphs if s >= count)
        with torch.cuda.stream(self.stream):
            self.inputs[:count].copy_(torch.from_numpy(host_inputs))
            self.graphs[size].replay()
            answers = self.outputs[size][:count].cpu()
        return answers.numpy()


def test_recorded_graphs_give_the_eager_bits(fry):
    network, _ = fry
    boards = random_boards(24, 5)
    with torch.no_grad():
        eager = network(torch.from_numpy(boards).long().cuda()).cpu().numpy()
    recorded = Recorded(network, torch.from_numpy(random_boards(24, 6)).long().cuda(), lane_sizes(24))
    assert np.array_equal(recorded.replay(boards), eager)
    assert np.array_equal(recorded.replay(boards[:10]), eager[:10])
    for _ in range(20):
        assert np.array_equal(recorded.replay(boards[:17]), eager[:17])


def test_the_engines_compiled_wrapping_records_and_replays_the_eager_bits(fry):
    # engine_search.network_graphs on capability (10, 0) (engine/engine_search.py:196-205) wraps the network in
    # ExactSizeCompiled (engine/inference.py:252-263): torch.compile(dynamic=False) for the chunk size and dynamic=True
    # for the rest, floats specialised; its runtime then records every size on a side stream, one private pool per lane.
    # The forward is the custom op fry::forward, which dynamo takes whole through its fake implementation.
    network, _ = fry
    chunk = 16
    exact, dynamic = torch.compile(network, dynamic=False), torch.compile(network, dynamic=True)

    def compiled(boards: torch.Tensor) -> torch.Tensor:
        with torch._dynamo.config.patch(specialize_float=True):
            return (exact if len(boards) == chunk else dynamic)(boards)

    boards = random_boards(chunk, 21)
    with torch.no_grad():
        eager = network(torch.from_numpy(boards).long().cuda()).cpu().numpy()
        assert np.array_equal(compiled(torch.from_numpy(boards).long().cuda()).cpu().numpy(), eager)
        assert np.array_equal(compiled(torch.from_numpy(boards[:5]).long().cuda()).cpu().numpy(), eager[:5])
    for _ in range(2):  # two lanes, each with its own graphs and pool
        recorded = Recorded(compiled, torch.from_numpy(random_boards(chunk, 22)).long().cuda(), [1, 2, 5, 8, chunk])
        assert np.array_equal(recorded.replay(boards), eager)
        assert np.array_equal(recorded.replay(boards[:5]), eager[:5])
        assert np.array_equal(recorded.replay(boards[:7]), eager[:7])


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


def lean_rows(boards: np.ndarray, seed: int) -> tuple[np.ndarray, np.ndarray]:
    """Lean lanes' rows (tokens, then int16 answer columns: a random number of distinct move columns, then the expected
    score's column as padding, as the Rust loop writes them) and those columns as int64."""
    rng = np.random.default_rng(seed)
    rows = np.zeros((len(boards), LEAN_ROW), dtype=np.uint8)
    rows[:, :TOKENS_PER_BOARD] = boards
    columns = np.full((len(boards), LEAN_COLUMNS), ANSWER_WIDTH - 1, dtype=np.int16)
    for b in range(len(boards)):
        legal = rng.integers(0, LEAN_COLUMNS)
        columns[b, :legal] = rng.choice(ANSWER_WIDTH - 1, size=legal, replace=False)
    rows[:, TOKENS_PER_BOARD:] = columns.astype("<i2").view(np.uint8).reshape(len(boards), -1)
    return rows, columns.astype(np.int64)


def test_lean_answers_are_the_rows_gathered_at_their_columns(fry):
    # engine/inference.py:130-135: a lean lane answers rows.gather(1, columns)
    network, _ = fry
    boards = random_boards(37, 8)
    rows_bytes, columns = lean_rows(boards, 8)
    with torch.no_grad():
        whole = network(torch.from_numpy(boards).long().cuda()).cpu()
        answers = network.forward_lean(torch.from_numpy(rows_bytes).cuda()).cpu()
    assert answers.shape == (37, LEAN_COLUMNS) and answers.dtype == torch.float32
    assert torch.equal(answers, whole.gather(1, torch.from_numpy(columns)))


def test_recorded_lean_graphs_give_the_eager_bits(fry):
    network, _ = fry
    boards = random_boards(24, 9)
    rows_bytes, _ = lean_rows(boards, 9)
    with torch.no_grad():
        eager = network.forward_lean(torch.from_numpy(rows_bytes).cuda()).cpu().numpy()
    start_rows, _ = lean_rows(random_boards(24, 10), 10)
    recorded = Recorded(network.forward_lean, torch.from_numpy(start_rows).cuda(), [8, 16, 24])
    assert np.array_equal(recorded.replay(rows_bytes), eager)
    assert np.array_equal(recorded.replay(rows_bytes[:10]), eager[:10])


def test_a_lean_column_outside_the_row_is_reported_not_faulted(fry):
    network, _ = fry
    lib = library()
    lib.device_status(clear=True)
    rows_bytes, _ = lean_rows(random_boards(3, 10), 10)
    rows_bytes[2, TOKENS_PER_BOARD + 2 * 5:TOKENS_PER_BOARD + 2 * 6] = np.array([ANSWER_WIDTH + 7], dtype="<i2").view(np.uint8)
    with torch.no_grad():
        answers = network.forward_lean(torch.from_numpy(rows_bytes).cuda())
    torch.cuda.synchronize()
    assert lib.device_status(clear=True) == (5, 2)
    assert answers[2, 5].item() == 0.0 and torch.isfinite(answers).all()


def test_fry_with_fp16_blocks_inside_and_last_runs_the_transitions(fry):
    # the engine's 26 + 2 layout: an fp16 block between int8 ones (each mixing its own input, link_input_mixes) and the
    # last; the fp16 blocks are the more exact, so the answers stay within int8's noise of the all-int8 network's
    network, _ = fry
    state = om.seeded_state_dict(FRY_SETTINGS, 1, std=0.02, template_std=0.02, table_std=0.02)
    weights = {layer: w for layer, w in oi.int8_weights(state, FRY_SETTINGS).items() if layer not in (13, 27)}
    mixed = Int8Network(state, FRY_SETTINGS, weights)
    assert [i for i, b in enumerate(mixed.blocks) if b["precision"] == 1] == [13, 27]
    boards = torch.from_numpy(random_boards(8, 12)).long().cuda()
    with torch.no_grad():
        ours, int8 = mixed(boards).cpu(), network(boards).cpu()
        alone = mixed(boards[[5]]).cpu()
    assert torch.isfinite(ours).all()
    assert (ours[:, :-1] - int8[:, :-1]).abs().max() <= 0.1 and (ours[:, -1] - int8[:, -1]).abs().max() <= 0.02
    assert torch.equal(alone, ours[[5]])  # an answer does not depend on its batch here either


def test_a_recorded_lean_graph_replays_by_its_raw_handle_as_the_rust_loop_does(fry):
    # the Rust round loop replays a lane's graph executable by raw handle on the lane's stream, between copies it makes
    # itself (engine/inference.py:175-205 spells the calls out in Python); here on a graph torch recorded
    import ctypes, os
    network, _ = fry
    rows_bytes, _ = lean_rows(random_boards(16, 13), 13)
    with torch.no_grad():
        eager = network.forward_lean(torch.from_numpy(rows_bytes).cuda()).cpu().numpy()
    start_rows, _ = lean_rows(random_boards(16, 14), 14)
    recorded = Recorded(network.forward_lean, torch.from_numpy(start_rows).cuda(), [8, 16])
    rows_host = torch.from_numpy(rows_bytes).pin_memory()
    answers_host = torch.zeros(16, LEAN_COLUMNS, dtype=torch.float32).pin_memory()
    stream = recorded.stream.cuda_stream
    cudart = ctypes.CDLL(f"libcudart.so.{torch.version.cuda.split('.')[0]}", mode=os.RTLD_NOLOAD | os.RTLD_LAZY)
    memcpy, launch, sync = cudart.cudaMemcpyAsync, cudart.cudaGraphLaunch, cudart.cudaStreamSynchronize
    memcpy.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_void_p]
    launch.argtypes, sync.argtypes = [ctypes.c_void_p] * 2, [ctypes.c_void_p]
    assert memcpy(recorded.inputs.data_ptr(), rows_host.data_ptr(), 16 * LEAN_ROW, 1, stream) == 0
    assert launch(recorded.graphs[16].raw_cuda_graph_exec(), stream) == 0
    assert memcpy(answers_host.data_ptr(), recorded.outputs[16].data_ptr(), 16 * LEAN_COLUMNS * 4, 2, stream) == 0
    assert sync(stream) == 0
    assert np.array_equal(answers_host.numpy(), eager)


def test_native_lanes_give_the_eager_bits(fry):
    # the C++ lane runtime (fry_lanes_*): the eager forward's bits, two batches out and collected in either order, and the
    # reference's refusals (engine/inference.py:167-171: RuntimeError with every lane busy)
    network, _ = fry
    boards = random_boards(24, 14)
    with torch.no_grad():
        eager = network(torch.from_numpy(boards).long().cuda()).cpu().numpy()
    batches = NativeBatches(network, lane_sizes(24), in_flight=2)
    try:
        first = batches.launch(boards[:10])
        second = batches.launch(boards)
        with pytest.raises(RuntimeError, match="more batches in flight than lanes"):
            batches.launch(boards[:3])
        assert np.array_equal(batches.collect(second), eager)
        assert np.array_equal(batches.collect(first), eager[:10])
        with pytest.raises(RuntimeError, match="no batch out"):
            batches.collect(first)
        with pytest.raises(RuntimeError, match="1 to 24 boards"):
            batches.launch_filled(batches.free_lane(), 25)
        for _ in range(20):
            assert np.array_equal(batches.collect(batches.launch(boards[:17])), eager[:17])
        batches.launch(boards[:5])
        batches.settle()
        assert all(not lane.pending for lane in batches.lanes)
    finally:
        batches.close()


def test_native_lean_lanes_give_the_eager_bits_and_replay_by_raw_handle(fry):
    # lean C++ lanes with blocking waits; then the Rust round loop's own calls on one of them, by raw handle through
    # torch's cudart (engine/inference.py:175-205): rows in, the size's graph, done, answers out
    import ctypes, os
    network, _ = fry
    boards = random_boards(24, 15)
    rows_bytes, _ = lean_rows(boards, 15)
    with torch.no_grad():
        eager = network.forward_lean(torch.from_numpy(rows_bytes).cuda()).cpu().numpy()
    batches = NativeBatches(network, [8, 16, 24], in_flight=2, blocking_wait=True, lean=True)
    try:
        with pytest.raises(RuntimeError, match="launch_filled"):
            batches.launch(boards)
        lane = batches.free_lane()
        lane.rows_array[:24] = rows_bytes
        first = batches.launch_filled(lane, 24)
        lane = batches.free_lane()
        lane.rows_array[:10] = rows_bytes[:10]
        second = batches.launch_filled(lane, 10)
        assert (first[1], second[1]) == (24, 16)
        assert np.array_equal(batches.collect(second), eager[:10])
        assert np.array_equal(batches.collect(first), eager)
        handles = batches.rust_network()["lanes"][1]
        cudart = ctypes.CDLL(f"libcudart.so.{torch.version.cuda.split('.')[0]}", mode=os.RTLD_NOLOAD | os.RTLD_LAZY)
        memcpy, launch, record, sync = cudart.cudaMemcpyAsync, cudart.cudaGraphLaunch, cudart.cudaEventRecord, cudart.cudaStreamSynchronize
        memcpy.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_void_p]
        launch.argtypes, record.argtypes, sync.argtypes = [ctypes.c_void_p] * 2, [ctypes.c_void_p] * 2, [ctypes.c_void_p]
        lane = batches.lanes[1]
        lane.rows_array[:16] = rows_bytes[8:]
        lane.answers_array[:] = 0
        executable, answers = handles["graphs"][16]
        assert memcpy(handles["rows"], handles["rows_host"], 16 * LEAN_ROW, 1, handles["stream"]) == 0
        assert launch(executable, handles["stream"]) == 0
        assert record(handles["done"], handles["stream"]) == 0
        assert memcpy(handles["answers_host"], answers, 16 * LEAN_COLUMNS * 4, 2, handles["stream"]) == 0
        assert sync(handles["stream"]) == 0
        assert np.array_equal(lane.answers_array[:16], eager[8:])
    finally:
        batches.close()
