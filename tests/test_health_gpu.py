"""The failure path of the kernels' bounded waits, made to run on the GPU without a fault: the device's wait limit is
lowered to 1 ms, a probe kernel waits on a barrier that nothing arrives at, and the wait runs out. The status word then
reads the timeout with the probe's site, the limit goes back, and the next forward is clean and gives the same answers
as before. The reference handles a failing kernel on the host (model/int8_cuda.py:370-381, tests/test_int8.py:187-199);
here the kernel itself gives up and says so."""
import ctypes
import time

import pytest
import torch

from chess_transformer_b200.boards import random_boards
from chess_transformer_b200.build import build
from chess_transformer_b200.library import library
from chess_transformer_b200.network import Int8Network
from oracle import int8 as oi, model as om
from tests.conftest import SMALL

pytestmark = pytest.mark.gpu

WAIT_TIMEOUT, PROBE_SITE = 1, 90
DEFAULT_LIMIT_NS = 2_000_000_000


@pytest.fixture(scope="module", autouse=True)
def built():
    build()


def wait_limit(lib) -> int:
    limit = ctypes.c_uint64()
    lib.fry_wait_limit_ns(ctypes.byref(limit))
    return limit.value


def test_a_wait_that_nothing_ends_runs_out_and_the_next_forward_is_clean():
    lib = library()
    state = om.seeded_state_dict(SMALL, 10)
    network = Int8Network(state, SMALL, oi.int8_weights(state, SMALL))
    boards = torch.from_numpy(random_boards(8, 4)).long().cuda()
    with torch.no_grad():
        before = network(boards)
    torch.cuda.synchronize()
    lib.device_status(clear=True)
    assert wait_limit(lib) == DEFAULT_LIMIT_NS
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    lib.fry_set_wait_limit_ns(1_000_000)
    try:
        assert wait_limit(lib) == 1_000_000
        start = time.perf_counter()
        lib.fry_wait_probe(stream)
        torch.cuda.synchronize()
        elapsed = time.perf_counter() - start
    finally:
        lib.fry_set_wait_limit_ns(DEFAULT_LIMIT_NS)
    assert lib.device_status(clear=True) == (WAIT_TIMEOUT, PROBE_SITE)
    assert 0.001 <= elapsed < 1.0  # the 1 ms limit, not the 2 s default
    assert wait_limit(lib) == DEFAULT_LIMIT_NS
    with torch.no_grad():
        after = network(boards)
    torch.cuda.synchronize()
    assert lib.device_status() == (0, 0)
    assert torch.equal(before, after)
