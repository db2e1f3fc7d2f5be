"""A profiling target: the 28-block int8 forward (or one of its kernels) between cudaProfilerStart and cudaProfilerStop,
so that `ncu --profile-from-start off` captures exactly that work. Warm-up runs happen before the start.

    ncu --profile-from-start off --metrics gpu__time_duration.sum --clock-control none --csv \\
        python chess-transformer_b200/profile_target.py --batch 256 --forwards 1
    ncu --profile-from-start off --set full --clock-control none -k regex:gemm_kernel -c 1 -o gpurun_out/gemm \\
        python chess-transformer_b200/profile_target.py --gemm gate_up --batch 256
"""
import argparse
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

# the int8 GEMMs of a block at M = batch x 70: (output columns N, depth K, gated)
GEMMS = {"projection": (1152, 768, False), "gate_up": (992, 768, True), "down": (768, 1024, False)}


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--batch", type=int, default=256)
    parser.add_argument("--forwards", type=int, default=1)
    parser.add_argument("--gemm", choices=sorted(GEMMS), help="profile one int8 GEMM launch instead of the forward")
    parser.add_argument("--warmup", type=int, default=2)
    args = parser.parse_args()

    import torch
    from chess_transformer_b200 import ops
    from chess_transformer_b200.boards import random_boards
    from chess_transformer_b200.network import FRY_SETTINGS, Int8Network, quantize, synthetic_state_dict

    torch.cuda.set_device(0)
    if args.gemm:
        N, K, gated = GEMMS[args.gemm]
        M = args.batch * 70
        generator = torch.Generator().manual_seed(0)
        x = torch.randint(-127, 128, (M, K), generator=generator, dtype=torch.int8).cuda()
        w = torch.randint(-127, 128, ((2 if gated else 1) * N, K), generator=generator, dtype=torch.int8).cuda()
        xs, ws = torch.rand(M).cuda() / 100, torch.rand(len(w)).cuda() / 100
        bias = torch.randn(N).half().cuda() if args.gemm == "projection" else None
        residual = torch.randn(M, N).half().cuda() if args.gemm == "down" else None
        run = lambda: ops.int8_linear(x, xs, w, ws, bias, residual, gated, args.gemm)
    else:
        state = synthetic_state_dict(FRY_SETTINGS, 0)
        network = Int8Network(state, FRY_SETTINGS, quantize(state, FRY_SETTINGS), "cuda:0")
        boards = torch.from_numpy(random_boards(args.batch, 0)).long().cuda()
        run = lambda: network(boards)
    with torch.no_grad():
        for _ in range(args.warmup):
            run()
        torch.cuda.synchronize()
        torch.cuda.profiler.start()
        for _ in range(args.forwards if not args.gemm else 1):
            run()
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()


if __name__ == "__main__":
    main()
