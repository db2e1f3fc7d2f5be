"""Benchmark of the Fry int8 forward on B200: positions/s of the 28-block network at batch 256 per GPU.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 --master-port P bench.py --gpus N

A step is one forward of 256 synthetic positions (seeded legal-looking boards, independent seeds per GPU) through the
full 28-block int8 network with random-init weights (no checkpoint ships here), replayed as a CUDA graph. Each GPU runs
its own replica: no collective on the data path and no NCCL at all (a gloo group on the host carries the barrier and the
max of the ranks' timings). L2 is flushed between timed steps by writing a 256 MiB buffer outside the timed events.
The end-to-end numbers go through the library's C++ lanes (fry_lanes_*, runtime.NativeBatches). Rank 0 prints one JSON
line.

--impl reference times the reference's own CPU implementation of the path, the fp32 ChessTransformer forward run through
cpu_batches (engine/inference.py:274-278), as restated by the CPU oracle (oracle/model.py), on all host cores: each step
one forward of the metric's 256 boards, or of a bounded sample of them when K + W such forwards would not end within
about three minutes.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

BATCH = 256
LATENCY_BATCH = 64
E2E_LANES = 2  # batches in flight in the end-to-end runs (the reference runtime's default, engine/inference.py:149)
CPU_SWEEP_BATCHES = (1, 16, 64, 256)  # the reference CPU path's batch sweep
REFERENCE_ARM_SECONDS = 180.0  # the reference arm's whole run stays within about this
# the library's kernels a forward launches: the embedding; per block 2 row norms, projection, attention, attention-out,
# gate_up, rotate_quant, down (8 x 28); the heads' final norm, f16 GEMM, narrow, policy, 2 x (split, sum), expected score
LAUNCHES_PER_FORWARD = 1 + 8 * 28 + 9
FLUSH_BYTES = 256 << 20
PROFILE_SUMMARY = ROOT / "profiles" / "int8_gemm_traffic.json"


def arguments():
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=20)
    parser.add_argument("--warmup", type=int, default=5)
    parser.add_argument("--impl", choices=["ours", "reference"], default="ours")
    parser.add_argument("--no-sweep", action="store_true", help="skip the batch sweep and the latency run")
    return parser.parse_args()


def peaks() -> dict:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        measured = json.loads(path.read_text())
        return {"hbm_gbs": measured["hbm_gbs"], "bf16_tflops": measured["bf16_tflops"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


def workload_config(world: int) -> dict:
    """The workload both arms measure (the reference arm on a bounded sample of it)."""
    return {"workload": "fry-28L-int8-forward-b256", "model": "fry d768, 28 blocks, 24q/12kv heads, dq 8/16/24, SwiGLU 992",
            "global_batch": BATCH * world, "seq_len": 70, "l2": "flushed between steps (256 MiB write outside the timed events)",
            "weights": "random-init N(0,0.02), round-to-nearest int8"}


class ClockSampler:
    """SM clock and clock-event (throttle) reasons sampled every 5 ms through NVML while the timed region runs (a
    reader only: it changes no setting); nvidia-smi every 200 ms where NVML is unavailable."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.device_index = device_index
        self.samples, self.max_mhz, self.source = [], None, None
        self.stop = threading.Event()
        self.thread = self.process = self.file = None
        self.nvml = self.handle = None

    def _read(self, nvml, handle):
        reasons = {"hw_slowdown": nvml.nvmlClocksEventReasonHwSlowdown, "hw_thermal_slowdown": nvml.nvmlClocksEventReasonHwThermalSlowdown,
                   "sw_thermal_slowdown": nvml.nvmlClocksEventReasonSwThermalSlowdown, "sw_power_cap": nvml.nvmlClocksEventReasonSwPowerCap}
        try:
            mhz = nvml.nvmlDeviceGetClockInfo(handle, nvml.NVML_CLOCK_SM)
            mask = nvml.nvmlDeviceGetCurrentClocksEventReasons(handle)
            self.samples.append((float(mhz), sorted(name for name, bit in reasons.items() if mask & bit)))
        except Exception:
            pass

    def _poll(self, nvml, handle):
        while not self.stop.is_set():
            self._read(nvml, handle)
            self.stop.wait(0.005)

    def sample_now(self) -> None:
        """One reading from the calling thread (the timed loop calls it after enqueueing each step, while the GPU runs the
        steps before): the polling thread may get few turns while the loop holds the interpreter."""
        if self.nvml is not None:
            self._read(self.nvml, self.handle)

    def __enter__(self):
        try:
            import pynvml as nvml
            nvml.nvmlInit()
            visible = os.environ.get("CUDA_VISIBLE_DEVICES")
            index = int(visible.split(",")[self.device_index]) if visible and visible.split(",")[0].isdigit() else self.device_index
            handle = nvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = float(nvml.nvmlDeviceGetMaxClockInfo(handle, nvml.NVML_CLOCK_SM))
            self.nvml, self.handle = nvml, handle
            self.thread = threading.Thread(target=self._poll, args=(nvml, handle), daemon=True)
            self.thread.start()
            self.source = "nvml, every 5 ms and once a step as it is enqueued"
        except Exception:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            try:
                self.process = subprocess.Popen(["nvidia-smi", f"--id={self.device_index}", f"--query-gpu={self.FIELDS}",
                                                 "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.file, stderr=subprocess.DEVNULL)
                self.source = "nvidia-smi, every 200 ms"
            except OSError:
                self.process = None
        return self

    def __exit__(self, *exc):
        self.stop.set()
        if self.thread is not None:
            self.thread.join(timeout=5)
        if self.process is not None:
            self.process.terminate()
            self.process.wait(timeout=10)

    def summary(self) -> dict:
        if self.file is not None:
            self.file.flush()
            self.file.seek(0)
            for row in (line.split(",") for line in self.file.read().splitlines() if line.strip()):
                if row[1].strip().replace(".", "").isdigit():
                    names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
                    self.samples.append((float(row[1]), sorted(n for n, v in zip(names, row[5:9]) if v.strip().lower() == "active")))
                    self.max_mhz = float(row[2]) if row[2].strip() else self.max_mhz
            Path(self.file.name).unlink(missing_ok=True)
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["no clock samples"], "samples": 0}
        return {"sm_mhz": statistics.median(mhz for mhz, _ in self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted({name for _, names in self.samples for name in names}), "samples": len(self.samples),
                "source": self.source}


def slowest_over_ranks(seconds: float) -> float:
    """The job's time: the largest of the ranks' times (an all_reduce MAX over the host-side gloo group), or the rank's
    own when it runs alone. Every rank calls it at the same point."""
    import torch
    import torch.distributed as dist
    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size() == 1:
        return seconds
    slowest = torch.tensor([seconds], dtype=torch.float64)
    dist.all_reduce(slowest, op=dist.ReduceOp.MAX)
    return slowest.item()


def host_cpu() -> str:
    """The host's CPU model, as /proc/cpuinfo names it."""
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_forward_seconds(torch, state: dict, settings: dict, boards, minimum_seconds: float, minimum_repeats: int) -> tuple[float, int]:
    """Mean seconds of the reference CPU path's fp32 forward (the oracle's restatement) on `boards`, after one untimed
    forward, over at least minimum_repeats forwards and minimum_seconds."""
    from oracle.model import fp32_forward
    with torch.no_grad():
        fp32_forward(state, settings, boards)
        start, repeats = time.perf_counter(), 0
        while repeats < minimum_repeats or time.perf_counter() - start < minimum_seconds:
            fp32_forward(state, settings, boards)
            repeats += 1
    return (time.perf_counter() - start) / repeats, repeats


def reference_arm(args, rank: int) -> None:
    """The reference's CPU path on the host cores: the fp32 forward of the metric's 256 boards a step, or of the largest
    halving of them whose K + W steps end within REFERENCE_ARM_SECONDS."""
    if rank != 0:
        return
    import torch
    from oracle.model import fp32_forward
    from chess_transformer_b200.boards import random_boards
    from chess_transformer_b200.network import FRY_SETTINGS, synthetic_state_dict
    torch.set_num_threads(os.cpu_count() or 1)
    state = synthetic_state_dict(FRY_SETTINGS, 0)
    sample = BATCH
    with torch.no_grad():
        while True:
            boards = torch.from_numpy(random_boards(sample, 0)).long()
            probe = time.perf_counter()
            fp32_forward(state, FRY_SETTINGS, boards)
            probe = time.perf_counter() - probe
            if sample == 1 or probe * (args.steps + args.warmup) <= REFERENCE_ARM_SECONDS:
                break
            sample //= 2
        for _ in range(max(0, args.warmup - 1)):
            fp32_forward(state, FRY_SETTINGS, boards)
        start = time.perf_counter()
        for _ in range(args.steps):
            fp32_forward(state, FRY_SETTINGS, boards)
        elapsed = time.perf_counter() - start
    value = sample * args.steps / elapsed
    cores = torch.get_num_threads()
    line = {"metric": "positions/sec (28L int8 fwd, batch 256)", "value": value, "unit": "positions/s", "impl": "reference",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * elapsed / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {**workload_config(1), "parallelism": "host cores",
                       "sample": f"{sample} of the batch's {BATCH} boards a step" + ("" if sample == BATCH else " (bounded CPU sample)")},
            "cpu_baseline": {"value": value, "unit": "positions/s", "cores": cores, "kind": "port",
                             "sample": f"{sample} boards x {args.steps} steps, fp32 ChessTransformer forward (oracle/model.py) "
                                       f"on {cores} threads, {os.cpu_count()} host cores ({host_cpu()})"},
            "e2e": {"value": value, "unit": "positions/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def cpu_baseline() -> dict:
    """The oracle port of the reference's CPU path on this host's cores at each of CPU_SWEEP_BATCHES (a few seconds a
    batch); the value is the metric's batch, 256."""
    import torch
    from chess_transformer_b200.boards import random_boards
    from chess_transformer_b200.network import FRY_SETTINGS, synthetic_state_dict
    threads = torch.get_num_threads()
    torch.set_num_threads(os.cpu_count() or 1)
    state = synthetic_state_dict(FRY_SETTINGS, 0)
    sweep, repeats_at = {}, {}
    for batch in CPU_SWEEP_BATCHES:
        boards = torch.from_numpy(random_boards(batch, 1)).long()
        seconds, repeats = cpu_forward_seconds(torch, state, FRY_SETTINGS, boards, 3.0, 2)
        sweep[str(batch)] = {"ms_per_forward": round(1000 * seconds, 2), "positions_per_s": round(batch / seconds, 2)}
        repeats_at[batch] = repeats
    cores = torch.get_num_threads()
    torch.set_num_threads(threads)
    return {"value": sweep[str(BATCH)]["positions_per_s"], "unit": "positions/s", "cores": cores, "kind": "port",
            "cpu": host_cpu(), "batch_sweep": sweep,
            "sample": f"the fp32 ChessTransformer forward (oracle/model.py, the reference's cpu_batches path) of "
                      f"{BATCH} boards x {repeats_at[BATCH]} forwards (and of {', '.join(str(b) for b in CPU_SWEEP_BATCHES[:-1])} "
                      f"boards for the sweep) on {cores} threads of {os.cpu_count()} host cores"}


def graphed(torch, stream, run):
    """run() recorded once into a CUDA graph on `stream` (after two eager warm-up calls); returns the graph's replay. A
    replay launches the kernel as the forward's graph does, so CUDA events around it time the kernel, not the host's
    argument checks and tensor-map encoding that precede an eager launch."""
    with torch.cuda.stream(stream):
        for _ in range(2):
            run()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            run()
    return graph.replay


def gemm_roofline(torch, stream) -> dict:
    """The dominant kernel, the int8 tensor-core GEMM, timed alone at the forward's shapes (M = 256 x 70 tokens, the
    launches of profile_target.GEMMS with their counts per forward): each recorded in a CUDA graph and replayed between
    CUDA events on its stream, L2 flushed before each replay: algorithmic int8 ops per launch / mean launch time,
    against the int8 dense peak."""
    from chess_transformer_b200 import ops
    from chess_transformer_b200.profile_target import GEMMS, gemm_runner
    M = BATCH * 70
    total_ops = total_seconds = 0.0
    per_shape = {}
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device="cuda")
    with torch.cuda.stream(stream):
        for name, (N, K, kind, count) in GEMMS.items():
            if kind == "fp16" or count == 0:
                continue
            run = graphed(torch, stream, gemm_runner(torch, ops, name, M))
            for _ in range(3):
                run()
            times = []
            for _ in range(10):
                flush.fill_(1)
                start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                start.record(stream)
                run()
                end.record(stream)
                end.synchronize()
                times.append(start.elapsed_time(end) / 1000)
            seconds = statistics.mean(times)
            ops_per_launch = 2.0 * M * K * N * (2 if kind.startswith("gated") else 1)
            per_shape[f"{name}_{N}x{K}"] = round(ops_per_launch / seconds / 1e12, 1)
            total_ops += ops_per_launch * count
            total_seconds += seconds * count
    return {"ops_per_forward": total_ops, "seconds_per_forward": total_seconds, "tops_by_shape": per_shape}


def timed_launches(torch, stream, flush, run, repeats: int = 10) -> float:
    """Mean seconds of run() on `stream` by CUDA events (replays of a CUDA graph of it), after 3 untimed launches, L2
    flushed before each timed one."""
    run = graphed(torch, stream, run)
    with torch.cuda.stream(stream):
        for _ in range(3):
            run()
        times = []
        for _ in range(repeats):
            flush.fill_(1)
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record(stream)
            run()
            end.record(stream)
            end.synchronize()
            times.append(start.elapsed_time(end) / 1000)
    return statistics.mean(times)


def microbench(torch, device, stream, flush) -> dict:
    """The benchmark's isolated-kernel configuration: the int8 GEMM with the per-row / per-column scale epilogue to bf16
    at each (K, N) and M it names (TOP/s against the int8 dense peak), and the seq-64 / head_dim-64 attention at 12 heads
    and batch 64 and 1024 (its HBM bytes, q, k, v read and out written, against the measured HBM peak); L2 flushed
    before each timed launch, operands seeded as the configuration says."""
    from chess_transformer_b200 import ops
    from oracle import microbench as mb
    peak = peaks()
    int8_peak = 2 * peak["bf16_tflops"]
    gemms = {}
    for K, N in mb.GEMM_SHAPES:
        for M in mb.GEMM_ROWS:
            x, weight, x_scale, weight_scale = (torch.from_numpy(a).to(device) for a in mb.gemm_operands(M, K, N, seed=M + K + N))
            seconds = timed_launches(torch, stream, flush, lambda: ops.int8_matmul_scaled_bf16(x, x_scale, weight, weight_scale))
            tops = 2.0 * M * K * N / seconds / 1e12
            gemms[f"M{M}_K{K}_N{N}"] = {"us": round(seconds * 1e6, 2), "tops": round(tops, 1), "frac": round(tops / int8_peak, 4)}
            del x, weight
    attention = {}
    for B in mb.ATTENTION_BATCHES:
        q, k, v = (t.to(device) for t in mb.attention_operands(B, seed=B))
        seconds = timed_launches(torch, stream, flush, lambda: ops.attention_bf16(q, k, v, mb.ATTENTION_HEADS))
        traffic = 4 * q.numel() * 2
        gbs = traffic / seconds / 1e9
        attention[str(B)] = {"us": round(seconds * 1e6, 2), "hbm_bytes": traffic, "gb_per_s": round(gbs, 1),
                             "hbm_frac": round(gbs / peak["hbm_gbs"], 4)}
    return {"gemm_int8_scaled_bf16": gemms, "attention_bf16_seq64_d64_h12": attention,
            "peaks": f"int8 dense = 2 x {peak['source']} bf16 burst ({int8_peak:.1f} TOP/s); HBM {peak['hbm_gbs']} GB/s, of {peak['source']}"}


SWEEP_BATCHES = (1, 16, 64, 256, 1024)
# batches also run as forwards of chunks, as the reference's chunked_answer_rows splits a batch so a chunk's activations
# stay in L2 (engine/inference.py:26-35): (batch, chunk)
SWEEP_CHUNKED = ((1024, 256), (1024, 128))
# HBM bytes a forward must read whatever the batch: the int8 block weights and the fp16 attention-out (28 blocks, dq
# cycling 8/16/24), for the small-batch regime's achieved GB/s
WEIGHT_BYTES = sum(768 * (36 * dq + 576) + 1984 * 768 + 768 * 1024 + 2 * 768 * 768 for dq in [8, 16, 24] * 9 + [8])


def batch_sweep(torch, network, device, stream, flush, steps: int) -> dict:
    """Positions/s and ms per forward at each of SWEEP_BATCHES, and at SWEEP_CHUNKED's batches run as forwards of chunks
    (a CUDA graph per batch, inputs resident, L2 flushed before each timed replay, CUDA events on the graph's stream).
    At batch 1 and 16 also the weights' achieved GB/s (WEIGHT_BYTES a forward) against the measured HBM peak."""
    from chess_transformer_b200.boards import random_boards
    results = {}
    hbm = peaks()["hbm_gbs"]
    for batch, chunk in [(batch, batch) for batch in SWEEP_BATCHES] + list(SWEEP_CHUNKED):
        boards = torch.from_numpy(random_boards(batch, 500 + batch)).long().to(device)
        parts = boards.split(chunk)
        with torch.cuda.stream(stream), torch.no_grad():
            for part in parts:
                network(part)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                for part in parts:
                    network(part)
            for _ in range(3):
                graph.replay()
            times = []
            for _ in range(steps):
                flush.fill_(1)
                start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                start.record(stream)
                graph.replay()
                end.record(stream)
                end.synchronize()
                times.append(start.elapsed_time(end))
        ms = statistics.median(times)
        entry = {"ms_per_forward": round(ms, 4), "positions_per_s": round(batch / ms * 1000, 1)}
        if batch <= 16:
            gbs = WEIGHT_BYTES / (ms / 1000) / 1e9
            entry.update({"weights_gb_per_s": round(gbs, 1), "hbm_frac": round(gbs / hbm, 4)})
        results[str(batch) if chunk == batch else f"{batch}_in_chunks_of_{chunk}"] = entry
        del graph
    return results


def main() -> None:
    args = arguments()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        reference_arm(args, rank)
        return

    import numpy as np
    import torch
    import torch.distributed as dist
    from chess_transformer_b200.boards import random_boards
    from chess_transformer_b200.network import FRY_SETTINGS, Int8Network, quantize, synthetic_state_dict
    from chess_transformer_b200.encoding import ANSWER_WIDTH, LEAN_COLUMNS, LEAN_ROW, TOKENS_PER_BOARD
    from chess_transformer_b200.runtime import NativeBatches

    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("gloo", timeout=timedelta(seconds=300))

    state = synthetic_state_dict(FRY_SETTINGS, 1000 + rank)
    network = Int8Network(state, FRY_SETTINGS, quantize(state, FRY_SETTINGS), device)
    del state
    boards = torch.from_numpy(random_boards(BATCH, 77 + rank)).long().to(device)
    stream = torch.cuda.Stream(device)
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=device)

    # the step as a CUDA graph (the reference records its forwards the same way, engine/inference.py:117-125)
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream), torch.no_grad():
        for _ in range(2):
            network(boards)
    torch.cuda.current_stream().wait_stream(stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream), torch.no_grad():
        rows = network(boards)
    torch.cuda.synchronize()
    if not torch.isfinite(rows).all():
        raise RuntimeError("the forward gave non-finite answers")

    with torch.cuda.stream(stream):
        for _ in range(max(3, args.warmup)):
            graph.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    with ClockSampler(local_rank) as clocks, torch.cuda.stream(stream):
        for start, end in events:
            flush.fill_(1)
            start.record(stream)
            graph.replay()
            end.record(stream)
            clocks.sample_now()
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    seconds = slowest_over_ranks(sum(start.elapsed_time(end) for start, end in events) / 1000)

    # end to end through the library's C++ lanes (fry_lanes_*): pinned host boards in, graph replay, answer rows out,
    # every step; two lanes, each step launched before the previous one is collected, as the reference's search keeps its
    # lanes in flight (engine/inference.py:144-146)
    def pipelined_seconds(launch, collect) -> float:
        def run(count: int) -> None:
            pending = launch()
            for _ in range(count - 1):
                following = launch()
                collect(pending)
                pending = following
            collect(pending)

        run(max(3, args.warmup))
        if world > 1:
            dist.barrier()
        start = time.perf_counter()
        run(args.steps)
        return slowest_over_ranks(time.perf_counter() - start)

    host_boards = random_boards(BATCH, 99 + rank)
    batches = NativeBatches(network, [LATENCY_BATCH, BATCH], in_flight=E2E_LANES)
    e2e_seconds = pipelined_seconds(lambda: batches.launch(host_boards), batches.collect)

    # the same through lean lanes, the Rust round loop's format: rows of tokens and answer columns in (30 moves' columns
    # a board, then the expected score's), 219 answers a board out
    lean_rows = np.zeros((BATCH, LEAN_ROW), dtype=np.uint8)
    lean_rows[:, :TOKENS_PER_BOARD] = host_boards
    columns = np.full((BATCH, LEAN_COLUMNS), ANSWER_WIDTH - 1, dtype="<i2")
    columns[:, :30] = np.random.default_rng(7 + rank).integers(0, ANSWER_WIDTH - 1, size=(BATCH, 30))
    lean_rows[:, TOKENS_PER_BOARD:] = columns.view(np.uint8).reshape(BATCH, -1)

    def lean_launch(runtime):
        lane = runtime.free_lane()
        lane.rows_array[:BATCH] = lean_rows
        return runtime.launch_filled(lane, BATCH)

    lean_batches = NativeBatches(network, [BATCH], in_flight=E2E_LANES, lean=True)
    lean_seconds = pipelined_seconds(lambda: lean_launch(lean_batches), lean_batches.collect)
    lean_batches.close()

    extra = {}
    if rank == 0 and not args.no_sweep:
        latencies = []
        for _ in range(60):
            t0 = time.perf_counter()
            batches.collect(batches.launch(host_boards[:LATENCY_BATCH]))
            latencies.append(time.perf_counter() - t0)
        extra["latency_p50_ms_batch64"] = round(1000 * statistics.median(latencies[10:]), 3)
    batches.close()
    if rank == 0 and not args.no_sweep:
        extra["batch_sweep"] = batch_sweep(torch, network, device, stream, flush, max(5, args.steps))

    if rank == 0:
        gemm = gemm_roofline(torch, stream)
        peak = peaks()
        int8_peak = 2 * peak["bf16_tflops"]
        achieved = gemm["ops_per_forward"] / gemm["seconds_per_forward"] / 1e12
        traffic = None
        if PROFILE_SUMMARY.exists():
            traffic = json.loads(PROFILE_SUMMARY.read_text()).get("dram_bytes_per_launch")
        roofline = {"bound": "tensor", "achieved": round(achieved, 1), "peak": round(int8_peak, 1), "unit": "TOP/s",
                    "frac": round(achieved / int8_peak, 4), "traffic": traffic,
                    "kernel": "gemm_kernel<kind::i8> (projection, gate_up, down at M=17920, weighted by launches per forward)",
                    "peak_source": f"int8 dense = 2 x {peak['source']} cuBLAS bf16 burst ({peak['bf16_tflops']} TFLOP/s), of {peak['source']}",
                    "tops_by_shape": gemm["tops_by_shape"]}
        forward_tops = 12.40e9 * BATCH / (seconds / args.steps) / 1e12
        line = {"metric": "positions/sec (28L int8 fwd, batch 256)", "value": BATCH * args.steps * world / seconds, "unit": "positions/s",
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * seconds / args.steps,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
                "config": {**workload_config(world), "parallelism": f"replicas x{world}"},
                "e2e": {"value": BATCH * args.steps * world / e2e_seconds, "unit": "positions/s",
                        "h2d_bytes_per_step": BATCH * 70 * 8, "d2h_bytes_per_step": BATCH * 1969 * 4, "lanes": E2E_LANES,
                        "runtime": "fry_lanes_* (C++ lanes: one C-ABI call to launch and one to collect)",
                        "note": "lanes on their own streams, a step launched before the previous one is collected; "
                                "no L2 flush between steps, unlike value"},
                "e2e_lean": {"value": BATCH * args.steps * world / lean_seconds, "unit": "positions/s",
                             "h2d_bytes_per_step": BATCH * LEAN_ROW, "d2h_bytes_per_step": BATCH * LEAN_COLUMNS * 4,
                             "runtime": "fry_lanes_* lean lanes (the Rust round loop's rows)"},
                "gpu_launches": LAUNCHES_PER_FORWARD * args.steps,
                "forward_int8_tops": round(forward_tops, 1),
                "roofline": roofline, "clocks": clocks.summary(), **extra}
        if not args.no_sweep:
            line["microbench"] = microbench(torch, device, stream, flush)
        if world == 1:
            line["cpu_baseline"] = cpu_baseline()
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
