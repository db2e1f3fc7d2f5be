"""The batch runtime around the network: CUDA graphs per batch size on lanes of their own stream, fed from pinned host
buffers. Mirrors the reference's `GraphedBatches` and `Lane` (engine/inference.py:62-225): `launch` copies a batch of
boards in and replays the smallest graph that holds it and returns at once; `collect` copies the answer rows out and
waits for them. At most `in_flight` batches are out at a time, one a lane. Lean lanes (lean=True, the Rust round loop's
format) take rows of tokens and answer columns through `free_lane().rows_array` and `launch_filled`, and `collect` gives
each board's LEAN_COLUMNS answers (the network's `forward_lean`), a ninth of the bytes of whole rows. `NativeBatches` is the
same runtime in the library's C++ (fry_lanes_*): no Python and no torch between a launch and its collect.
"""
import ctypes

import numpy as np
import torch
from torch import nn

from .boards import START_BOARD
from .encoding import ANSWER_WIDTH, LEAN_COLUMNS, LEAN_ROW, TOKENS_PER_BOARD
from .library import FryError, FryLaneHandles, library


def small_graph_sizes(max_batch: int, chunk: int | None = None) -> list[int]:
    """engine/inference.py:62-68: sizes 1..max_batch, doubling to 16, then steps of a sixteenth."""
    chunk = min(chunk or max_batch, max_batch)
    steps = [1]
    while steps[-1] < chunk:
        steps.append(min(chunk, steps[-1] * 2 if steps[-1] < 16 else steps[-1] + max(4, steps[-1] // 16)))
    sizes = [whole + step for whole in range(0, max_batch, chunk) for step in steps]
    return sizes[:next(index for index, size in enumerate(sizes) if size >= max_batch) + 1]


class Lane:
    """One stream with a graph per size, its own memory pool, and pinned buffers for the boards in and the rows out. A lean
    lane takes rows of LEAN_ROW bytes (tokens, then int16 answer columns, all 1968 at first: the expected score's) and
    answers LEAN_COLUMNS floats a board (engine/inference.py:94-106)."""

    def __init__(self, model: nn.Module, sizes: list[int], lean: bool = False):
        self.stream = torch.cuda.Stream()
        self.device = torch.cuda.current_device()
        self.pending = False
        self.lean = lean
        largest = sizes[-1]
        # recorded on real boards, as the reference records its lanes
        self.boards = torch.from_numpy(np.tile(START_BOARD, (largest, 1))).long().cuda()
        if lean:
            self.rows = torch.zeros(largest, LEAN_ROW, dtype=torch.uint8, device="cuda")
            self.rows[:, :TOKENS_PER_BOARD] = self.boards
            self.rows[:, TOKENS_PER_BOARD:].view(torch.int16).fill_(ANSWER_WIDTH - 1)
            self.rows_host = torch.zeros(largest, LEAN_ROW, dtype=torch.uint8, pin_memory=True)
            self.rows_array = self.rows_host.numpy()
        else:
            self.boards_host = torch.zeros(largest, TOKENS_PER_BOARD, dtype=torch.long, pin_memory=True)
            self.boards_array = self.boards_host.numpy()
        self.answers_host = torch.zeros(largest, LEAN_COLUMNS if lean else ANSWER_WIDTH, dtype=torch.float32, pin_memory=True)
        self.answers_array = self.answers_host.numpy()
        self.done = torch.cuda.Event(blocking=True)
        answer = (lambda size: model.forward_lean(self.rows[:size])) if lean else (lambda size: model(self.boards[:size]))
        self.stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(self.stream), torch.no_grad():
            for size in sizes:
                answer(size)
        torch.cuda.current_stream().wait_stream(self.stream)
        self.pool = torch.cuda.graph_pool_handle()
        self.graphs, self.answers = {}, {}
        for size in reversed(sizes):
            self.graphs[size] = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graphs[size], pool=self.pool, stream=self.stream), torch.no_grad():
                self.answers[size] = answer(size)
        self.done.record(self.stream)  # the event's handle exists from its first record
        self.done.synchronize()

    def handles(self) -> dict:
        """The raw handles a caller outside Python replays the lane with (engine/inference.py:138-142): the device, the
        stream and done event, the rows' pinned and device buffers, the answers' pinned buffer, and for each size its graph's
        executable and answers on the device."""
        return {"device": self.device, "stream": self.stream.cuda_stream, "done": self.done.cuda_event,
                "rows_host": self.rows_host.data_ptr(), "rows": self.rows.data_ptr(), "answers_host": self.answers_host.data_ptr(),
                "graphs": {size: (graph.raw_cuda_graph_exec(), self.answers[size].data_ptr()) for size, graph in self.graphs.items()}}


class GraphedBatches:
    """engine/inference.py:148-225: launch(boards uint8/int64 [n, 70]) -> handle; collect(handle) -> float32 [n, 1969]. Lean
    (lean=True): fill free_lane().rows_array[:n], launch_filled(lane, n), collect(handle) -> float32 [n, 219]."""

    def __init__(self, model: nn.Module, sizes: list[int], in_flight: int = 2, blocking_wait: bool = False, lean: bool = False):
        self.model, self.sizes, self.blocking_wait, self.lean = model, sizes, blocking_wait, lean
        self.lanes = [Lane(model, sizes, lean) for _ in range(in_flight)]
        self.handles = {id(lane): lane.handles() for lane in self.lanes} if lean else {}

    def rust_network(self) -> dict:
        """engine/inference.py:207-211: what the Rust round loop (Searches) replays the lean lanes with, no Python between
        rounds; it calls the CUDA runtime by these handles as it does the reference's lanes."""
        if not self.lean:
            raise ValueError("Searches' round loop needs lean lanes")
        return {"blocking_wait": self.blocking_wait, "lanes": [self.handles[id(lane)] for lane in self.lanes]}

    def free_lane(self) -> Lane:
        lane = next((lane for lane in self.lanes if not lane.pending), None)
        if lane is None:
            raise RuntimeError("more batches in flight than lanes")
        return lane

    def launch(self, boards: np.ndarray) -> tuple[Lane, int, int]:
        if self.lean:
            raise RuntimeError("lean lanes answer rows with their columns (launch_filled), not boards")
        lane = self.free_lane()
        lane.boards_host[:len(boards)] = torch.from_numpy(np.asarray(boards))
        return self.launch_filled(lane, len(boards))

    def launch_filled(self, lane: Lane, count: int) -> tuple[Lane, int, int]:
        size = next(size for size in self.sizes if size >= count)
        lane.pending = True
        with torch.cuda.stream(lane.stream):
            if lane.lean:
                lane.rows[:count].copy_(lane.rows_host[:count], non_blocking=True)
            else:
                lane.boards[:count].copy_(lane.boards_host[:count], non_blocking=True)
            lane.graphs[size].replay()
            if self.blocking_wait:
                lane.done.record(lane.stream)
        return lane, size, count

    def collect(self, launched: tuple[Lane, int, int]) -> np.ndarray:
        lane, size, count = launched
        if self.blocking_wait:
            lane.done.synchronize()
        with torch.cuda.stream(lane.stream):
            lane.answers_host[:count].copy_(lane.answers[size][:count])
        lane.stream.synchronize()
        lane.pending = False
        return lane.answers_host[:count].numpy()

    def settle(self) -> None:
        for lane in self.lanes:
            if lane.pending:
                lane.stream.synchronize()
                lane.pending = False


class NativeLane:
    """A lane of NativeBatches: its index and numpy views of its pinned buffers (boards_array, or a lean lane's rows_array,
    and answers_array), as `Lane` has them."""

    def __init__(self, index: int, handles: FryLaneHandles, largest: int, lean: bool):
        self.index, self.handles, self.lean, self.pending = index, handles, lean, False
        if lean:
            self.rows_array = np.ctypeslib.as_array(ctypes.cast(handles.rows_host, ctypes.POINTER(ctypes.c_uint8)), shape=(largest, LEAN_ROW))
        else:
            self.boards_array = np.ctypeslib.as_array(ctypes.cast(handles.rows_host, ctypes.POINTER(ctypes.c_int64)),
                                                      shape=(largest, TOKENS_PER_BOARD))
        width = LEAN_COLUMNS if lean else ANSWER_WIDTH
        self.answers_array = np.ctypeslib.as_array(ctypes.cast(handles.answers_host, ctypes.POINTER(ctypes.c_float)), shape=(largest, width))


class NativeBatches:
    """`GraphedBatches` (engine/inference.py:148-225) over the library's C++ lanes: fry_lanes_create records the network's
    forward (fry_forward, or fry_forward_lean for lean lanes) into a CUDA graph per size on each lane, on the current
    device; launch/launch_filled/collect/settle/free_lane/rust_network behave as the reference's, with the lane calls in
    C++. The network is kept alive: the graphs read its weights where they were recorded. close() frees the lanes."""

    def __init__(self, network: nn.Module, sizes: list[int], in_flight: int = 2, blocking_wait: bool = False, lean: bool = False):
        self.network, self.sizes, self.blocking_wait, self.lean = network, list(sizes), blocking_wait, lean
        self._lib = library()
        handle = ctypes.c_void_p()
        self._lib.fry_lanes_create(ctypes.byref(network._network), (ctypes.c_int * len(sizes))(*sizes), len(sizes), in_flight, int(lean),
                                   int(blocking_wait), ctypes.byref(handle))
        self._lanes = handle
        self.lanes = []
        for index in range(in_flight):
            handles = FryLaneHandles()
            self._lib.fry_lanes_handles(self._lanes, index, ctypes.byref(handles))
            self.lanes.append(NativeLane(index, handles, self.sizes[-1], lean))
        if self.lanes[0].handles.device != torch.cuda.current_device():
            device = self.lanes[0].handles.device
            self.close()
            raise FryError(f"the lanes were made on device {device}, not on torch's current device {torch.cuda.current_device()}")

    def free_lane(self) -> NativeLane:
        index = ctypes.c_int()
        self._lib.fry_lanes_free_lane(self._lanes, ctypes.byref(index))
        return self.lanes[index.value]

    def launch(self, boards: np.ndarray) -> tuple[NativeLane, int, int]:
        if self.lean:
            raise RuntimeError("lean lanes answer rows with their columns (launch_filled), not boards")
        lane = self.free_lane()
        lane.boards_array[:len(boards)] = np.asarray(boards)
        return self.launch_filled(lane, len(boards))

    def launch_filled(self, lane: NativeLane, count: int) -> tuple[NativeLane, int, int]:
        size = ctypes.c_int()
        self._lib.fry_lanes_launch(self._lanes, lane.index, count, ctypes.byref(size))
        lane.pending = True
        return lane, size.value, count

    def collect(self, launched: tuple[NativeLane, int, int]) -> np.ndarray:
        lane, _, count = launched
        self._lib.fry_lanes_collect(self._lanes, lane.index, None)
        lane.pending = False
        return lane.answers_array[:count]

    def settle(self) -> None:
        self._lib.fry_lanes_settle(self._lanes)
        for lane in self.lanes:
            lane.pending = False

    def rust_network(self) -> dict:
        """engine/inference.py:207-211: the lanes' raw handles, every size's graph writing the lane's one answers buffer."""
        if not self.lean:
            raise ValueError("Searches' round loop needs lean lanes")
        lanes = []
        for lane in self.lanes:
            h = lane.handles
            graphs = {}
            for index, size in enumerate(self.sizes):
                executable = ctypes.c_void_p()
                self._lib.fry_lanes_graph(self._lanes, lane.index, index, ctypes.byref(executable))
                graphs[size] = (executable.value, h.answers)
            lanes.append({"device": h.device, "stream": h.stream, "done": h.done, "rows_host": h.rows_host, "rows": h.rows,
                          "answers_host": h.answers_host, "graphs": graphs})
        return {"blocking_wait": self.blocking_wait, "lanes": lanes}

    def close(self) -> None:
        if getattr(self, "_lanes", None):
            self._lib.fry_lanes_destroy(self._lanes)
            self._lanes = None

    def __del__(self):
        self.close()
