"""The batch runtime around the network, in the library's C++ (fry_lanes_*): per lane a stream, a CUDA graph of the
forward per batch size, pinned host buffers for the boards in and the answers out, and a done event, with no Python and
no torch between a launch and its collect. `NativeBatches` is its Python face, with the method names the reference's
search calls on its own runtime (`GraphedBatches`, engine/inference.py:148-225): `launch` copies a batch of boards in,
replays the smallest graph that holds it and returns at once; `collect` copies the answer rows out and waits for them.
Lean lanes (lean=True, the Rust round loop's format) take rows of tokens and answer columns through
`free_lane().rows_array` and `launch_filled`, and `collect` gives each board's LEAN_COLUMNS answers (the network's
`forward_lean`), a ninth of the bytes of whole rows.

The reference's own `GraphedBatches` needs none of this: it records `Int8Network.forward` into its graphs unchanged.
"""
import ctypes

import numpy as np
import torch
from torch import nn

from .encoding import ANSWER_WIDTH, LEAN_COLUMNS, LEAN_ROW, TOKENS_PER_BOARD
from .library import FryError, FryLaneHandles, library


def lane_sizes(largest: int, coarse_from: int = 16) -> list[int]:
    """Batch sizes to record a graph for, ascending, ending at `largest`: every power of two below `coarse_from`, then
    multiples of coarse_from / 2, so a batch replays a graph at most coarse_from / 2 - 1 boards (or a power of two)
    larger than itself."""
    sizes, size = [], 1
    while size < min(largest, coarse_from):
        sizes.append(size)
        size *= 2
    step = max(1, coarse_from // 2)
    size = max(size, step)
    while size < largest:
        sizes.append(size)
        size += step
    sizes.append(largest)
    return sorted(set(sizes))


class NativeLane:
    """A lane of NativeBatches: its index and numpy views of its pinned buffers (boards_array, or a lean lane's rows_array,
    and answers_array), views that stay valid while the lanes live."""

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
