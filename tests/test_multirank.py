"""The multi-GPU path's host logic on CPU ranks (no GPU): the job's time is the slowest rank's, taken by an all_reduce MAX
over a world-size-2 gloo group (bench.py uses the same host-side group on the GPUs: no NCCL); and under torchrun the
reference arm runs on rank 0 alone, which prints the one JSON line, while the other rank exits 0 without work."""
import json
import os
import socket
import subprocess
import sys

import torch.distributed as dist
import torch.multiprocessing as mp

from tests.conftest import ROOT

sys.path.insert(0, str(ROOT))
import bench  # noqa: E402


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def slowest_worker(rank: int, world: int, port: int, times: list[float], results) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        results.put((rank, bench.slowest_over_ranks(times[rank])))
    finally:
        dist.destroy_process_group()


def test_the_job_time_is_the_slowest_ranks_over_two_gloo_ranks():
    context = mp.get_context("spawn")
    results = context.Queue()
    times, port = [0.75, 1.25], free_port()
    processes = [context.Process(target=slowest_worker, args=(rank, 2, port, times, results)) for rank in range(2)]
    for process in processes:
        process.start()
    found = dict(results.get(timeout=120) for _ in processes)
    for process in processes:
        process.join(timeout=60)
        assert process.exitcode == 0
    assert found == {0: 1.25, 1: 1.25}


def test_a_rank_alone_keeps_its_own_time():
    assert not dist.is_initialized()
    assert bench.slowest_over_ranks(0.5) == 0.5


def test_the_reference_arm_runs_on_rank_zero_alone_under_torchrun():
    command = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2", "--master-addr", "127.0.0.1",
               "--master-port", str(free_port()), str(ROOT / "bench.py"), "--impl", "reference", "--gpus", "2", "--steps", "1",
               "--warmup", "0"]
    done = subprocess.run(command, capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert done.returncode == 0, done.stderr[-2000:]
    lines = [json.loads(line) for line in done.stdout.splitlines() if line.startswith("{")]
    assert len(lines) == 1
    line = lines[0]
    assert line["impl"] == "reference" and line["n_gpus"] == 2 and line["value"] > 0
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["cpu_baseline"]["kind"] == "port"
