"""GPTQ on the device: drop-ins for the reference's `gptq` (engine/quantization.py:76-99), `input_hessians` (:103-119),
`compute_int8_weights` (:122-140), `block_errors` (:144-169), the ranking that picks the blocks kept in fp16, and
`int8_weights` (:188-207), a checkpoint's int8 weights read from the cache or computed and cached.
fry_gptq rounds a matmul's weights in fp64 on its GPU, and fry_hessian_accumulate sums the inputs x^T x that its Hessian
is made of; the answers are the reference's Int8Weights.
"""
import ctypes
import hashlib
import os
import sys
from contextlib import suppress
from pathlib import Path

import torch
from torch import nn

from .calibration import CalibrationNetwork
from .encoding import NUM_MOVE_IDS, TOKENS_PER_BOARD
from .library import FryError, library
from .network import DOWN_INPUT_MULTIPLE, FP16_LAST_LAYERS, HADAMARD_BLOCK, Int8Network, down_inputs, geometry, hadamard, load_checkpoint

# The cache of computed int8 weights, shared with the reference's engine: the same folder (its environment variable, else
# ~/.cache/chess_transformer/int8) and, for the reference's own calibration, the same file names, so the weights the
# reference cached for a checkpoint load here unchanged (engine/quantization.py:26-48,174-185).
CACHE_VARIABLE = "CHESS_TRANSFORMER_INT8_CACHE"
# what the reference's cached files are named by: its rounding code's version, its calibration (1024 positions of its
# PGN from game 1000, every 9th ply), GPTQ's dampening and column block, the blocks kept fp16 at the end, the down's
# rotation and padding, and for a choice of fp16 blocks the choice's version and count
REFERENCE_ROUNDING = (1, 1024, 1000, 9, 0.01, 128, FP16_LAST_LAYERS, HADAMARD_BLOCK, DOWN_INPUT_MULTIPLE)
CHOICE_VERSION = 1

NOT_POSITIVE_DEFINITE = 6  # the device status code fry_gptq records


def gptq(weight: torch.Tensor, hessian: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """engine/quantization.py:76-99: (int8 weight, fp32 scale a row) of an N x K weight, each column's error spread over
    the later ones through the Hessian [K, K]. Both are taken as fp64 (as the reference takes them) on the weight's CUDA
    device. Raises FryError if the dampened Hessian is not positive definite, where the reference's
    torch.linalg.cholesky raises."""
    if weight.dim() != 2 or hessian.shape != (weight.shape[1], weight.shape[1]):
        raise ValueError(f"gptq takes weight [N, K] and hessian [K, K], got {tuple(weight.shape)} and {tuple(hessian.shape)}")
    device = weight.device if weight.is_cuda else torch.device("cuda")
    weight64 = weight.detach().to(device=device, dtype=torch.float64).contiguous()
    hessian64 = hessian.detach().to(device=device, dtype=torch.float64).contiguous()
    N, K = weight64.shape
    lib = library()
    integers = torch.empty(N, K, dtype=torch.int8, device=device)
    scale = torch.empty(N, dtype=torch.float32, device=device)
    workspace = torch.empty(lib.fry_gptq_workspace_bytes(N, K), dtype=torch.uint8, device=device)
    with torch.cuda.device(device):
        before = lib.device_status()
        stream = torch.cuda.current_stream(device)
        lib.fry_gptq(ctypes.c_void_p(weight64.data_ptr()), ctypes.c_void_p(hessian64.data_ptr()), N, K,
                     ctypes.c_void_p(integers.data_ptr()), ctypes.c_void_p(scale.data_ptr()), ctypes.c_void_p(workspace.data_ptr()),
                     workspace.numel(), ctypes.c_void_p(stream.cuda_stream))
        stream.synchronize()
        code, where = lib.device_status()
        if code == NOT_POSITIVE_DEFINITE and before[0] != NOT_POSITIVE_DEFINITE:
            lib.device_status(clear=True)
            raise FryError(f"gptq: the dampened Hessian is not positive definite (Cholesky pivot {where})")
    return integers, scale


@torch.no_grad()
def input_hessians(model: nn.Module, boards: torch.Tensor, batch: int = 128) -> list[dict[str, torch.Tensor]]:
    """engine/quantization.py:103-119: per block of `model` (the reference's ChessTransformer, or any module with its
    `encoder` blocks and their Q, mlp.gate_projection and mlp.down_projection), the fp64 sum over the boards' tokens of
    x^T x for the inputs x of its projection, gate_up and down matmuls, summed on the GPU by fry_hessian_accumulate."""
    lib = library()
    device = next(model.parameters()).device
    device = device if device.type == "cuda" else torch.device("cuda")
    hessians = [{} for _ in model.encoder]
    hooks = []
    for block, sums in zip(model.encoder, hessians):
        for name, layer in (("projection", block.Q), ("gate_up", block.mlp.gate_projection), ("down", block.mlp.down_projection)):
            def add(module, inputs, name=name, sums=sums):
                x = inputs[0].reshape(-1, inputs[0].shape[-1]).to(device=device, dtype=torch.float64).contiguous()
                if name not in sums:
                    sums[name] = torch.zeros(x.shape[1], x.shape[1], dtype=torch.float64, device=device)
                lib.fry_hessian_accumulate(ctypes.c_void_p(x.data_ptr()), x.shape[0], x.shape[1], ctypes.c_void_p(sums[name].data_ptr()),
                                           ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream))
            hooks.append(layer.register_forward_pre_hook(add))
    try:
        for start in range(0, len(boards), batch):
            model(boards[start:start + batch].to(next(model.parameters()).device))
    finally:
        for hook in hooks:
            hook.remove()
    torch.cuda.synchronize(device)
    return hessians


def gptq_inputs(state: dict, layer: int, sums: dict[str, torch.Tensor]) -> dict[str, tuple[torch.Tensor, torch.Tensor]]:
    """engine/quantization.py:129-139: a block's (weight, hessian) pairs as gptq takes them, fp64 on the sums' device:
    projection = Q|K|V|template mix rows with the projection's sums; gate_up = gate rows then up rows with gate_up's; down
    zero-padded to a multiple of 128 inputs and rotated, weight = pad(W) R / 32 and hessian = R^T pad(H) R, R the
    block-diagonal 32 x 32 Hadamard matrix. `state` is named as the reference's ChessTransformer names its weights."""
    device = sums["down"].device
    p = f"encoder.{layer}."
    w = lambda name: state[p + name].to(device=device, dtype=torch.float64)
    projection = torch.cat([w(n + ".weight") for n in ("Q", "K", "V", "template_mix")])
    gate_up = torch.cat([w("mlp.gate_projection.weight"), w("mlp.up_projection.weight")])
    hidden = state[p + "mlp.down_projection.weight"].shape[1]
    width = down_inputs(hidden)
    padding = width - hidden
    rotation = torch.block_diag(*[hadamard(HADAMARD_BLOCK)] * (width // HADAMARD_BLOCK)).to(device=device, dtype=torch.float64)
    padded = nn.functional.pad(sums["down"].double(), (0, padding, 0, padding))
    down = nn.functional.pad(w("mlp.down_projection.weight"), (0, padding)) @ rotation / HADAMARD_BLOCK
    return {"projection": (projection, sums["projection"].double()), "gate_up": (gate_up, sums["gate_up"].double()),
            "down": (down, rotation.t() @ padded @ rotation)}


def int8_weights_from_sums(state: dict, hessians: list[dict[str, torch.Tensor]], layers: list[int] | None = None) -> dict:
    """Int8Weights {layer: {"projection"|"gate_up"|"down": (int8 [N, K], fp32 [N])}} of a state dict from input_hessians'
    sums, every block but the last FP16_LAST_LAYERS by default (engine/quantization.py:126), each matmul rounded by GPTQ
    on the device."""
    layers = range(len(hessians) - FP16_LAST_LAYERS) if layers is None else layers
    return {layer: {name: gptq(weight, hessian) for name, (weight, hessian) in gptq_inputs(state, layer, hessians[layer]).items()}
            for layer in layers}


@torch.no_grad()
def compute_int8_weights(model: nn.Module, boards: torch.Tensor) -> dict:
    """engine/quantization.py:122-140, same signature: the Int8Weights of `model` (the reference's ChessTransformer,
    loaded as int8_weights loads it, :200-201) calibrated on `boards`, every block but the last."""
    return int8_weights_from_sums(model.state_dict(), input_hessians(model, boards))


@torch.no_grad()
def block_errors(state: dict, settings: dict, weights: dict, boards: torch.Tensor, legal: torch.Tensor, batch: int = 256) -> dict[int, float]:
    """engine/quantization.py:144-169: per block of `weights`, the mean over the boards of the total variation between
    the policy (softmax over each board's legal moves, fp64) of the fp16 network and of the fp16 network with only that
    block in int8. Both networks run through fry_forward (Int8Network with the one block's weights, or none). boards int64
    [n, 70] and legal bool [n, 1968] are the calibration positions and their legal moves, which the reference reads from
    its PGN through python-chess."""
    device = torch.device("cuda", torch.cuda.current_device())
    boards, legal = boards.to(device), legal.to(device=device, dtype=torch.bool)

    def priors(int8_layers: list[int]) -> torch.Tensor:
        network = Int8Network(state, settings, {layer: weights[layer] for layer in int8_layers}, device)
        logits = torch.cat([network(boards[start:start + batch])[:, :-1] for start in range(0, len(boards), batch)])
        return torch.softmax(logits.double().masked_fill(~legal, -torch.inf), dim=-1)

    fp16 = priors([])
    return {layer: 0.5 * (priors([layer]) - fp16).abs().sum(dim=-1).mean().item() for layer in weights}


def fp16_choice(errors: dict[int, float], fp16_blocks: int) -> list[int]:
    """engine/quantization.py:196-198: the fp16_blocks blocks of the largest block_errors, which stay fp16."""
    return sorted(errors, key=errors.get, reverse=True)[:fp16_blocks]


def cache_folder() -> Path | None:
    """The weights cache's folder: $CHESS_TRANSFORMER_INT8_CACHE, else ~/.cache/chess_transformer/int8; None without
    either (engine/quantization.py:29-35)."""
    if os.environ.get(CACHE_VARIABLE):
        return Path(os.environ[CACHE_VARIABLE])
    try:
        return Path.home() / ".cache" / "chess_transformer" / "int8"
    except RuntimeError:
        return None


def calibration_digest(boards: torch.Tensor, legal: torch.Tensor | None = None) -> str:
    """sha256 of the calibration positions' tokens (and legal-move masks, when given), naming weights calibrated on them."""
    digest = hashlib.sha256(boards.detach().to(device="cpu", dtype=torch.int64).contiguous().numpy().tobytes())
    if legal is not None:
        digest.update(legal.detach().to(device="cpu", dtype=torch.bool).contiguous().numpy().tobytes())
    return digest.hexdigest()


def cached_weights_path(checkpoint_path: Path, fp16_blocks: int, calibration: str | None = None) -> Path | None:
    """The cache file of a checkpoint's int8 weights: named by the checkpoint's sha256 and a digest of how they were
    rounded. With calibration None, the reference's own name for its own calibration (engine/quantization.py:174-185);
    with a calibration digest, the same name with that digest among the rounding's settings, so weights calibrated on
    other positions never pass for the reference's."""
    folder = cache_folder()
    if folder is None:
        return None
    with open(checkpoint_path, "rb") as checkpoint:
        digest = hashlib.file_digest(checkpoint, "sha256").hexdigest()
    rounding = REFERENCE_ROUNDING + ((CHOICE_VERSION, fp16_blocks) if fp16_blocks else ())
    if calibration is not None:
        rounding += ("calibration", calibration)
    return folder / f"{digest}_{hashlib.sha256(repr(rounding).encode()).hexdigest()[:16]}.pt"


def save_cached_weights(weights: dict, path: Path | None) -> None:
    """Written under another name and renamed, so engines starting together never read half a file; a cache that cannot
    be written only costs the next start its time (engine/quantization.py:211-224)."""
    if path is None:
        print("the int8 weights are not cached: there is no cache folder", file=sys.stderr)
        return
    partial = path.with_name(f"{path.name}.{os.getpid()}.partial")
    try:
        path.parent.mkdir(parents=True, exist_ok=True)
        torch.save(weights, partial)
        os.replace(partial, path)
    except (OSError, RuntimeError) as error:
        with suppress(OSError):
            partial.unlink()
        print(f"the int8 weights are not cached: {error}", file=sys.stderr)


def int8_weights(checkpoint_path: Path, fp16_blocks: int, calibration: tuple[torch.Tensor, torch.Tensor | None] | None = None,
                 device: torch.device | str | None = None) -> dict:
    """engine/quantization.py:188-207: the checkpoint's Int8Weights on the CPU, every block in int8 but the last and the
    fp16_blocks blocks of the largest block_errors.

    calibration None: the weights the reference cached for this checkpoint (its own calibration on its PGN's positions,
    under its own file name), or FryError if it has none. calibration (boards int64 [n, 70], legal bool [n, 1968] or
    None): weights calibrated on those positions, read from the cache or computed on `device` (GPTQ over the fp64
    network's input Hessians, then, for fp16_blocks > 0, block_errors over the positions' legal moves) and cached."""
    if fp16_blocks < 0:
        raise ValueError(f"a count of blocks to keep in fp16, not {fp16_blocks}")
    checkpoint_path = Path(checkpoint_path)
    if calibration is None:
        path = cached_weights_path(checkpoint_path, fp16_blocks)
        if path is not None and path.exists():
            return torch.load(path, weights_only=True)
        raise FryError(f"no cached int8 weights for {checkpoint_path} with {fp16_blocks} more fp16 blocks, and no calibration positions to "
                       "compute them: pass calibration=(boards [n, 70], legal [n, 1968]) (the reference reads 1024 positions of its PGN "
                       "through python-chess), or the weights themselves")
    boards, legal = calibration if isinstance(calibration, (tuple, list)) else (calibration, None)
    boards = torch.as_tensor(boards)
    if boards.dim() != 2 or boards.shape[1] != TOKENS_PER_BOARD:
        raise FryError(f"calibration boards are [n, {TOKENS_PER_BOARD}] tokens, got {tuple(boards.shape)}")
    if fp16_blocks and (legal is None or tuple(legal.shape) != (boards.shape[0], NUM_MOVE_IDS)):
        raise FryError(f"choosing {fp16_blocks} fp16 blocks needs the calibration positions' legal moves, bool [n, {NUM_MOVE_IDS}]")
    path = cached_weights_path(checkpoint_path, fp16_blocks, calibration_digest(boards, legal if fp16_blocks else None))
    if path is not None and path.exists():
        return torch.load(path, weights_only=True)
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    state, settings = load_checkpoint(checkpoint_path)
    if fp16_blocks:
        weights = int8_weights(checkpoint_path, 0, (boards, None), device)
        errors = block_errors(state, settings, weights, boards, legal)
        kept = fp16_choice(errors, fp16_blocks)
        weights = {layer: matmuls for layer, matmuls in weights.items() if layer not in kept}
    else:
        with torch.cuda.device(device):
            model = CalibrationNetwork(state, geometry(settings), device)
            weights = {layer: {name: tuple(tensor.cpu() for tensor in pair) for name, pair in matmuls.items()}
                       for layer, matmuls in int8_weights_from_sums(state, input_hessians(model, boards)).items()}
            del model
    save_cached_weights(weights, path)
    return weights
