"""fry_heads_noalloc: the heads for callers that cannot allocate device memory (a thread in the middle of a stream
capture, a latency-bound loop that must not risk an allocation's device-wide synchronisation, or a host in another
language without a device allocator), against fry_heads with a caller-provided workspace.

The entry point keeps its scratch in a fixed device array inside the library, shared by every call on a device, so it
takes at most FRY_HEADS_NOALLOC_MAX_BOARDS boards of d_model up to FRY_HEADS_NOALLOC_MAX_D_MODEL. This file is named to
be collected last, so that a run stopping at the first failure has run every other test first; it also passes alone.
"""
import ctypes

import pytest
import torch

from chess_transformer_b200.build import build
from chess_transformer_b200.library import FryError, library
from chess_transformer_b200.ops import heads_struct
from oracle import int8 as oi, model as om

pytestmark = pytest.mark.gpu

MAX_BOARDS, MAX_D_MODEL = 16, 768


def prepared_heads(d_model: int):
    settings = {"d_model": d_model, "num_layers": 1, "n_heads": d_model // 32, "kv_heads": d_model // 64, "qk_ratio": [0.5],
                "mlp_hidden": 2 * d_model, "value_bins": 128}
    state = om.seeded_state_dict(settings, 21, from_scale=8.0)
    prepared = oi.prepare(state, settings, oi.int8_weights(state, settings))
    weights = [prepared["ln"], prepared["a_weight"].t().contiguous(), prepared["a_bias"], prepared["narrow_weight"], prepared["narrow_bias"],
               prepared["eval_head.0.weight"], prepared["eval_head.0.bias"], prepared["eval_head.2.weight"], prepared["eval_head.2.bias"]]
    return [tensor.cuda().contiguous() for tensor in weights]


def rows_with_workspace(lib, stream_x, weights, struct):
    B, _, D = stream_x.shape
    rows = torch.empty(B, 1969, device="cuda")
    workspace = torch.empty(lib.fry_heads_workspace_bytes(B, D), device="cuda", dtype=torch.uint8)
    lib.fry_heads(ctypes.c_void_p(stream_x.data_ptr()), ctypes.byref(struct), 1e-5, ctypes.c_void_p(rows.data_ptr()),
                  ctypes.c_void_p(workspace.data_ptr()), workspace.numel(), B, D, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    return rows


def rows_without_workspace(lib, stream_x, struct):
    B, _, D = stream_x.shape
    rows = torch.empty(B, 1969, device="cuda")
    lib.fry_heads_noalloc(ctypes.c_void_p(stream_x.data_ptr()), ctypes.byref(struct), 1e-5, ctypes.c_void_p(rows.data_ptr()), B, D,
                          ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    return rows


@pytest.fixture(scope="module", autouse=True)
def built():
    build()


def test_the_allocation_free_heads_give_the_heads_answers_on_two_calls_in_a_row():
    lib = library()
    weights = prepared_heads(MAX_D_MODEL)
    struct = heads_struct(*weights)
    generator = torch.Generator().manual_seed(3)
    # two calls in a row on different boards: the second finds the first call's contents in the shared array
    for boards in (MAX_BOARDS, 5):
        stream_x = (torch.randn(boards, 70, MAX_D_MODEL, generator=generator) / 4).half().cuda()
        found = rows_without_workspace(lib, stream_x, struct)
        expected = rows_with_workspace(lib, stream_x, weights, struct)
        torch.cuda.synchronize()
        # the same kernels on the same inputs: the tolerance the heads tests use is met with no difference at all
        assert torch.equal(found, expected), boards
        assert torch.isfinite(found).all()


def test_the_allocation_free_heads_replay_from_a_captured_graph():
    # the header's contract: one call outside a capture (it sets the kernels' attributes), then the entry point records
    # into a CUDA graph on a side stream with no allocation, and every replay writes the heads' answers
    lib = library()
    weights = prepared_heads(MAX_D_MODEL)
    struct = heads_struct(*weights)
    stream_x = (torch.randn(8, 70, MAX_D_MODEL, generator=torch.Generator().manual_seed(5)) / 4).half().cuda()
    expected = rows_with_workspace(lib, stream_x, weights, struct)
    rows = torch.empty(8, 1969, device="cuda")
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    call = lambda: lib.fry_heads_noalloc(ctypes.c_void_p(stream_x.data_ptr()), ctypes.byref(struct), 1e-5, ctypes.c_void_p(rows.data_ptr()),
                                         8, MAX_D_MODEL, ctypes.c_void_p(side.cuda_stream))
    with torch.cuda.stream(side):
        call()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            call()
    torch.cuda.current_stream().wait_stream(side)
    for _ in range(2):
        rows.zero_()
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(rows, expected)


def test_the_allocation_free_heads_refuse_more_than_their_array_holds():
    lib = library()
    weights = prepared_heads(MAX_D_MODEL)
    struct = heads_struct(*weights)
    stream_x = torch.zeros(MAX_BOARDS + 1, 70, MAX_D_MODEL, dtype=torch.float16, device="cuda")
    with pytest.raises(FryError, match="at most 16 boards"):
        rows_without_workspace(lib, stream_x, struct)


@pytest.mark.parametrize("d_model", [MAX_D_MODEL + 16, 0, -16, 40])
def test_the_allocation_free_heads_refuse_a_width_they_do_not_take(d_model):
    lib = library()
    struct = heads_struct(*prepared_heads(MAX_D_MODEL))
    stream_x = torch.zeros(2, 70, MAX_D_MODEL, dtype=torch.float16, device="cuda")
    rows = torch.empty(2, 1969, device="cuda")
    with pytest.raises(FryError, match="d_model"):
        lib.fry_heads_noalloc(ctypes.c_void_p(stream_x.data_ptr()), ctypes.byref(struct), 1e-5, ctypes.c_void_p(rows.data_ptr()), 2, d_model,
                              ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
