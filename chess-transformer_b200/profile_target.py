"""A profiling target: the 28-block int8 forward (or its GEMMs alone) between cudaProfilerStart and cudaProfilerStop, so
that `ncu --profile-from-start off` captures exactly that work. Warm-up runs happen before the start.

    ncu --profile-from-start off --metrics gpu__time_duration.sum --clock-control none --csv \\
        python chess-transformer_b200/profile_target.py --batch 256 --forwards 1
    ncu --profile-from-start off --set full --clock-control none -k regex:gemm_kernel -c 1 -o gemm \\
        python chess-transformer_b200/profile_target.py --gemm gate_up --batch 256
    ncu --profile-from-start off --metrics dram__bytes_read.sum,dram__bytes_write.sum --clock-control none \\
        -k regex:gemm_kernel --csv python chess-transformer_b200/profile_target.py --gemm all --batch 256
"""
import argparse
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

# the GEMMs of a block at M = batch x 70: name -> (output columns N, depth K, kind), and how many of the 28 blocks run
# each: the projection at dq 8/16/24 (at dq 8 and 16 with the attention's q/k norm in its epilogue, "bias_qk"), gate_up,
# down mixing the next block's input (the last block's adds its residual only), and the attention-out fp16 linear; then
# the GEMMs with the norm in their prologue (kinds "_normed"), which the forward does not run (count 0), for profiling
# them beside the others
GEMMS = {"projection864": (864, 768, "bias_qk", 10), "projection1152": (1152, 768, "bias_qk", 9), "projection1440": (1440, 768, "bias", 9),
         "gate_up": (992, 768, "gated", 28), "down": (768, 1024, "mixing", 27), "down_last": (768, 1024, "residual", 1),
         "combine": (768, 768, "fp16", 28), "projection1152_normed": (1152, 768, "bias_normed", 0),
         "gate_up_normed": (992, 768, "gated_normed", 0)}


def gemm_runner(torch, ops, name: str, M: int):
    N, K, kind, _ = GEMMS[name]
    generator = torch.Generator().manual_seed(0)
    if kind == "fp16":
        x = torch.randn(M, K, generator=generator).half().cuda()
        weight = (torch.randn(N, K, generator=generator) / 16).half().cuda()  # [N, K]: the layout the library takes
        bias = torch.randn(N, generator=generator).half().cuda()
        residual = torch.randn(M, N, generator=generator).half().cuda()
        out = torch.empty(M, N, dtype=torch.half, device="cuda")
        from chess_transformer_b200 import library
        return lambda: library().fry_linear(x.data_ptr(), weight.data_ptr(), bias.data_ptr(), residual.data_ptr(), out.data_ptr(), M, N,
                                            K, 0, torch.cuda.current_stream().cuda_stream)
    gated = kind.startswith("gated")
    if kind.endswith("_normed"):
        x = (torch.randn(M, K, generator=generator) * 3).half().cuda()
        gain = (torch.rand(K, generator=generator) + 0.5).half().cuda()
        w = torch.randint(-127, 128, ((2 if gated else 1) * N, K), generator=generator, dtype=torch.int8).cuda()
        ws = (torch.rand(len(w), generator=generator) / 100).cuda()
        bias = None if gated else torch.randn(N, generator=generator).half().cuda()
        return lambda: ops.int8_linear_normed(x, gain, 1e-5, w, ws, bias, gated)
    x = torch.randint(-127, 128, (M, K), generator=generator, dtype=torch.int8).cuda()
    w = torch.randint(-127, 128, ((2 if gated else 1) * N, K), generator=generator, dtype=torch.int8).cuda()
    xs, ws = (torch.rand(M, generator=generator) / 100).cuda(), (torch.rand(len(w), generator=generator) / 100).cuda()
    bias = torch.randn(N, generator=generator).half().cuda() if kind.startswith("bias") else None
    if kind == "bias_qk":  # Fry's projection rows: 24 query heads, 12 key heads of dq = (N - 576) / 36
        import ctypes
        from chess_transformer_b200 import library
        dq = (N - 576) // 36
        gains = (1 + torch.randn(2, dq, generator=generator) / 10).half().cuda()
        out = torch.empty(M, N, dtype=torch.half, device="cuda")
        pointer = lambda tensor: ctypes.c_void_p(tensor.data_ptr())
        return lambda: library().fry_int8_linear_qk_norm(pointer(x), pointer(xs), pointer(w), pointer(ws), pointer(bias), pointer(gains[0]),
                                                         pointer(gains[1]), 1e-5, pointer(out), M, N, K, 24, 12, dq,
                                                         ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    residual = torch.randn(M, N, generator=generator).half().cuda() if kind in ("residual", "mixing") else None
    mix = ()
    if kind == "mixing":
        mix = (torch.randn(M, N, generator=generator).half().cuda(), torch.tensor([0.8]).half().cuda(), torch.tensor([0.5]).half().cuda())
    return lambda: ops.int8_linear(x, xs, w, ws, bias, residual, gated, name, *mix)


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--batch", type=int, default=256)
    parser.add_argument("--forwards", type=int, default=1)
    parser.add_argument("--gemm", choices=sorted(GEMMS) + ["all"], help="profile GEMM launches instead of the forward "
                        "(all: one launch of each, in the order of GEMMS)")
    parser.add_argument("--warmup", type=int, default=2)
    args = parser.parse_args()

    import torch
    from chess_transformer_b200 import ops
    from chess_transformer_b200.boards import random_boards
    from chess_transformer_b200.network import FRY_SETTINGS, Int8Network, quantize, synthetic_state_dict

    torch.cuda.set_device(0)
    if args.gemm:
        names = list(GEMMS) if args.gemm == "all" else [args.gemm]
        runners = [gemm_runner(torch, ops, name, args.batch * 70) for name in names]
        run_all = lambda: [run() for run in runners]
        runs = 1
    else:
        state = synthetic_state_dict(FRY_SETTINGS, 0)
        network = Int8Network(state, FRY_SETTINGS, quantize(state, FRY_SETTINGS), "cuda:0")
        boards = torch.from_numpy(random_boards(args.batch, 0)).long().cuda()
        run_all = lambda: network(boards)
        runs = args.forwards
    with torch.no_grad():
        for _ in range(args.warmup):
            run_all()
        torch.cuda.synchronize()
        torch.cuda.profiler.start()
        for _ in range(runs):
            run_all()
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()


if __name__ == "__main__":
    main()
