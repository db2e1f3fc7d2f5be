"""Host-side checks that need no GPU: the C-ABI library builds, loads and exports every entry point include/fry_b200.h
declares; the product's move table, weight layout and synthetic boards agree with the oracle; CPU tensors are refused."""
import ctypes
import re
import subprocess
from pathlib import Path

import numpy as np
import pytest
import torch

import chess_transformer_b200 as fry
from chess_transformer_b200 import boards as fry_boards, encoding as fry_encoding, network as fry_network
from chess_transformer_b200.build import build
from chess_transformer_b200.library import LIBRARY_PATH, SIGNATURES, FryError, FryHeads, library
from oracle import encoding, int8 as oi, model as om
from tests.conftest import ROOT, SMALL

HEADER = ROOT / "include" / "fry_b200.h"


def declared_functions() -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(fry_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    build()
    return library()


def test_the_library_exports_every_declared_entry_point(lib):
    declared = declared_functions()
    assert len(declared) >= 15
    exported = subprocess.run(["nm", "-D", "--defined-only", str(LIBRARY_PATH)], capture_output=True, text=True, check=True).stdout
    names = {line.split()[-1] for line in exported.splitlines() if line.strip()}
    assert set(declared) <= names
    assert set(declared) == set(SIGNATURES)
    assert lib.fry_version().decode().startswith("fry_b200")


def test_the_library_is_built_for_sm_100a_only():
    from chess_transformer_b200.build import FLAGS
    assert "arch=compute_100a,code=sm_100a" in FLAGS and sum(flag.startswith("arch=") for flag in FLAGS) == 1


def test_shapes_are_refused_on_the_host_before_any_launch(lib):
    with pytest.raises(FryError, match="multiple of 8"):
        lib.fry_int8_linear(None, None, None, None, None, None, None, None, None, None, 70, 12, 256, 0, None)
    with pytest.raises(FryError, match="K = 768"):
        lib.fry_int8_linear_normed(None, None, 1e-5, None, None, None, None, 70, 864, 512, 0, None)
    with pytest.raises(FryError, match="multiple of 256"):
        lib.fry_linear_norm_quant(None, None, None, None, None, None, 1e-5, None, None, 70, 800, 768, None)
    with pytest.raises(FryError, match="template attention"):
        lib.fry_template_attention(None, None, None, None, None, 1, 24, 12, 8, 64, 8, 1e-5, None)
    assert "template attention" in lib.fry_last_error().decode()
    # the fused projection and attention take query/key heads 8 or 16 wide, their blocks on 16-column boundaries, or 24
    # wide on 48-column boundaries
    for dq, heads in ((24, 23), (8, 3), (32, 24), (12, 24)):
        with pytest.raises(FryError, match="8 or 16 wide"):
            lib.fry_int8_linear_qk_norm(None, None, None, None, None, None, None, 1e-5, None, 70, 1440, 768, heads, 12, dq, None)
    with pytest.raises(FryError, match="dq 8, 16 or 24"):
        lib.fry_template_attention_normed(None, None, None, 1, 24, 12, 32, 32, 8, None)
    for limit in (0, 999, 60_000_000_001):
        with pytest.raises(FryError, match="1 us to 60 s"):
            lib.fry_set_wait_limit_ns(limit)
    with pytest.raises(FryError, match="d_model"):
        lib.fry_heads(None, ctypes.byref(FryHeads()), 1e-5, None, None, 0, 2, 0, None)


def test_the_ops_refuse_cpu_tensors():
    from chess_transformer_b200 import ops
    x = torch.zeros(2, 70, 128, dtype=torch.float16)
    with pytest.raises(FryError, match="GPU only"):
        ops.norm_quant(x, torch.ones(128, dtype=torch.float16), 1e-5)


def test_the_move_table_is_the_oracles():
    assert fry_encoding.NUM_MOVE_IDS == encoding.NUM_MOVE_IDS == 1968
    assert np.array_equal(fry_encoding.MOVE_FROM_SQUARES, encoding.MOVE_FROM_SQUARES)
    assert np.array_equal(fry_encoding.MOVE_TO_SQUARES, encoding.MOVE_TO_SQUARES)
    promotions = np.full(1968, -1)
    promotions[encoding.PROMOTION_MOVE_IDS] = encoding.PROMOTION_PIECES
    assert np.array_equal(fry_encoding.MOVE_PROMOTION_PIECES, promotions)


def test_the_compiled_move_table_is_current():
    assert (ROOT / "chess-transformer_b200" / "csrc" / "moves.h").read_text() == fry_encoding.moves_header()


def test_the_weight_layout_is_the_oracles():
    state = om.seeded_state_dict(SMALL, 10)
    ours, theirs = fry_network.quantize(state, SMALL), oi.int8_weights(state, SMALL)
    for layer in theirs:
        for name in ("projection", "gate_up", "down"):
            assert torch.equal(ours[layer][name][0], theirs[layer][name][0])
            assert torch.equal(ours[layer][name][1], theirs[layer][name][1])


def test_synthetic_boards_are_legal_looking_and_seeded():
    boards = fry_boards.random_boards(512, 7)
    assert boards.shape == (512, 70) and boards.dtype == np.uint8
    assert np.array_equal(boards, fry_boards.random_boards(512, 7))
    assert not np.array_equal(boards, fry_boards.random_boards(512, 8))
    squares = boards[:, :64]
    assert ((squares == 6).sum(1) == 1).all() and ((squares == 12).sum(1) == 1).all()
    others = ((squares > 0) & (squares != 6) & (squares != 12)).sum(1)
    assert others.min() >= 2 and others.max() <= 30
    assert not np.isin(squares[:, :8], [1, 7]).any() and not np.isin(squares[:, 56:], [1, 7]).any()
    assert np.isin(boards[:, 64], [13, 14]).all() and np.isin(boards[:, 65:69], [15, 16]).all()
    assert ((boards[:, 69] == 17) | ((boards[:, 69] >= 57) & (boards[:, 69] < 65))).all()
    # the oracle's square features take them
    om.square_feature_indices(torch.from_numpy(boards[:8]))


def test_start_board_is_the_initial_position():
    start = fry_boards.START_BOARD
    assert start[4] == 6 and start[60] == 12 and (start[8:16] == 1).all() and (start[48:56] == 7).all() and start[64] == 14


def test_the_synthetic_checkpoint_loads_into_the_oracles_shapes():
    state = fry_network.synthetic_state_dict(SMALL, 0)
    shapes = om.parameter_shapes(SMALL)
    assert set(shapes) == set(state)
    assert all(tuple(state[name].shape) == shape for name, shape in shapes.items())


def test_int8_model_without_weights_needs_a_cache_or_calibration_positions(tmp_path, monkeypatch):
    from chess_transformer_b200 import quantization
    monkeypatch.setenv(quantization.CACHE_VARIABLE, str(tmp_path / "cache"))
    torch.save({"model_settings": SMALL, "state_dict": om.seeded_state_dict(SMALL, 0)}, tmp_path / "model.pt")
    for blocks in (0, 1):
        with pytest.raises(FryError, match="calibration"):
            quantization.int8_weights(tmp_path / "model.pt", blocks)
    with pytest.raises(FryError, match="legal moves"):
        quantization.int8_weights(tmp_path / "model.pt", 1, (torch.zeros(4, 70, dtype=torch.long), None))
    with pytest.raises(ValueError, match="count of blocks"):
        quantization.int8_weights(tmp_path / "model.pt", -1)
    with pytest.raises(FryError, match="CUDA"):
        fry_network.int8_model(tmp_path / "model.pt", device="cpu")


def test_the_weights_cache_is_named_as_the_references(tmp_path, monkeypatch):
    # engine/quantization.py:174-185: <sha256 of the checkpoint>_<16 hex of the rounding settings>.pt under the cache
    # folder, so the weights the reference cached load unchanged; weights calibrated on other positions get other names
    import hashlib
    from chess_transformer_b200 import quantization
    monkeypatch.setenv(quantization.CACHE_VARIABLE, str(tmp_path))
    checkpoint = tmp_path / "model.pt"
    checkpoint.write_bytes(b"checkpoint bytes")
    digest = hashlib.sha256(b"checkpoint bytes").hexdigest()
    rounding = (1, 1024, 1000, 9, 0.01, 128, 1, 32, 128)
    assert quantization.cached_weights_path(checkpoint, 0) == tmp_path / f"{digest}_{hashlib.sha256(repr(rounding).encode()).hexdigest()[:16]}.pt"
    with_choice = rounding + (1, 2)
    assert quantization.cached_weights_path(checkpoint, 2).name == f"{digest}_{hashlib.sha256(repr(with_choice).encode()).hexdigest()[:16]}.pt"
    ours = quantization.cached_weights_path(checkpoint, 0, quantization.calibration_digest(torch.zeros(2, 70, dtype=torch.long)))
    assert ours.name.startswith(digest) and ours != quantization.cached_weights_path(checkpoint, 0)


def test_the_forward_ops_have_fake_implementations_for_torch_compile():
    # dynamo traces the forward through these (the reference's custom ops register fakes the same way,
    # model/int8_blocks.py:141-144); no GPU is touched
    from torch._subclasses.fake_tensor import FakeTensorMode
    import chess_transformer_b200.network  # noqa: F401  (registers fry::forward and fry::forward_lean)
    with FakeTensorMode():
        rows = torch.ops.fry.forward(torch.empty(5, 70, dtype=torch.int64), 1)
        answers = torch.ops.fry.forward_lean(torch.empty(3, fry_encoding.LEAN_ROW, dtype=torch.uint8), 1)
    assert rows.shape == (5, fry_encoding.ANSWER_WIDTH) and rows.dtype == torch.float32
    assert answers.shape == (3, fry_encoding.LEAN_COLUMNS) and answers.dtype == torch.float32


def test_the_lean_row_format_is_the_rust_loops():
    # engine/selfplay_rs/src/lib.rs:330-333
    assert (fry_encoding.LEGAL_SLOTS, fry_encoding.LEAN_COLUMNS, fry_encoding.LEAN_ROW) == (218, 219, 508)


def test_lean_forward_is_refused_on_the_host_without_a_network(lib):
    with pytest.raises(FryError, match="needs a network"):
        lib.fry_forward_lean(None, None, 4, None, None, 0, None)
    assert lib.fry_forward_lean_workspace_bytes(None, 4) == 0


def test_lane_calls_are_refused_on_the_host_before_any_cuda_call(lib):
    # fry_lanes_*: the batch runtime's argument checks come before its first CUDA call, so they run without a GPU
    import ctypes
    from chess_transformer_b200.library import ERROR_SHAPE, FryNetwork
    network, handle = FryNetwork(), ctypes.c_void_p()
    sizes = lambda *s: (ctypes.c_int * len(s))(*s)
    with pytest.raises(FryError, match="ascending"):
        lib.fry_lanes_create(ctypes.byref(network), sizes(1, 8, 4), 3, 2, 0, 0, ctypes.byref(handle))
    with pytest.raises(FryError, match="ascending"):
        lib.fry_lanes_create(ctypes.byref(network), sizes(0, 4), 2, 2, 1, 0, ctypes.byref(handle))
    with pytest.raises(FryError, match="at least one size and one lane"):
        lib.fry_lanes_create(ctypes.byref(network), sizes(1, 2), 2, 0, 0, 0, ctypes.byref(handle))
    assert handle.value is None
    raw = lib.handle
    assert raw.fry_lanes_free_lane(None, None) == ERROR_SHAPE and "needs lanes" in raw.fry_last_error().decode()
    assert raw.fry_lanes_launch(None, 0, 1, None) == ERROR_SHAPE and "no such lane" in raw.fry_last_error().decode()
    assert raw.fry_lanes_collect(None, 0, None) == ERROR_SHAPE
    assert raw.fry_lanes_destroy(None) == 0


def test_the_header_is_plain_c_and_a_c_program_links_the_library(lib, tmp_path):
    # a host written in C (or bound through any C FFI) sees exactly include/fry_b200.h: it compiles as C11, and its
    # refusals come back through the C ABI before any CUDA call, so this runs without a GPU
    source = tmp_path / "host.c"
    source.write_text(r"""
#include <stdio.h>
#include <string.h>
#include "fry_b200.h"

int main(void) {
    int sizes[2] = {8, 4};
    FryNetwork network;
    FryLanes* lanes = NULL;
    memset(&network, 0, sizeof network);
    int status;
    printf("%s\n", fry_version());
    status = fry_lanes_create(&network, sizes, 2, 1, 1, 0, &lanes);
    printf("%d %s\n", status, fry_last_error());
    status = fry_gptq(NULL, NULL, 8, 128, NULL, NULL, NULL, 0, NULL);
    printf("%d %s\n", status, fry_last_error());
    printf("%d %d\n", FRY_LEAN_ROW, FRY_LEAN_COLUMNS);
    return lanes != NULL;
}
""")
    binary = tmp_path / "host"
    subprocess.run(["gcc", "-std=c11", "-Wall", "-Werror", "-I", str(HEADER.parent), str(source), "-o", str(binary),
                    "-L", str(LIBRARY_PATH.parent), "-lfry_b200", f"-Wl,-rpath,{LIBRARY_PATH.parent}"], check=True)
    out = subprocess.run([str(binary)], capture_output=True, text=True, check=True).stdout.splitlines()
    assert out[0].startswith("fry_b200")
    assert out[1].startswith("1 ") and "ascending" in out[1]
    assert out[2].startswith("1 ") and "needs its weight" in out[2]
    assert out[3] == "508 219"
