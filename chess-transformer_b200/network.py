"""The int8 network as the engine's search sees it: the drop-in for the reference's `engine.inference.int8_model`.

`int8_model(checkpoint_path, fp16_blocks, weights)` (engine/inference.py:267-272) loads a checkpoint in the reference's
format (`{"model_settings", "state_dict"}`, model/checkpoint.py:22-42) and int8 weights in the reference's
`Int8Weights` layout (engine/quantization.py:21,124-140), and returns an `Int8Network` whose
`forward(boards: LongTensor[B, 70] cuda) -> Tensor[B, 1969] fp32` gives the answer rows that `answer_rows`
(engine/inference.py:19-23) would give, and which has `.d_model` (engine/engine_search.py:198).

Set-up follows `fp16_model` and `quantize_blocks` (engine/inference.py:242-249, model/int8_blocks.py:254-298): the residual
stream is scaled by 1/16 (embedding tables, combine_heads, down's scale), everything but the heads is fp16, the heads'
weights are folded in fp64 (model/fused_blocks.py:815-824). The whole forward is one C-ABI call (fry_forward) that
enqueues every kernel on the current stream, so the module records into CUDA graphs like the reference's.
"""
import ctypes
import itertools
import math
import weakref
from pathlib import Path

import numpy as np
import torch
from torch import nn

from .encoding import ANSWER_WIDTH, BOARD_VOCAB_SIZE, FEATURE_TABLE_ROWS, LEAN_COLUMNS, LEAN_ROW, TOKENS_PER_BOARD, VALUE_TOKEN_DIM
from .library import BLOCK_FP16, BLOCK_INT8, FryBlock, FryError, FryNetwork, library
from .ops import heads_struct, pair_templates

FP16_RESIDUAL_SCALE = 1 / 16      # engine/inference.py:239
HADAMARD_BLOCK = 32               # model/int8_blocks.py:15
DOWN_INPUT_MULTIPLE = 128         # model/int8_blocks.py:17
INT8_MAX = 127                    # engine/quantization.py:47
EPS = 1e-5

# Fry's shipped geometry (fry-final-117): 28 blocks, d 768, 24 query heads of 32, 12 key/value heads, SwiGLU 992 wide,
# 128 value bins; the query/key width cycles 8/16/24 over the blocks
FRY_SETTINGS = {"d_model": 768, "num_layers": 28, "n_heads": 24, "kv_heads": 12, "qk_ratio": [0.25, 0.5, 0.75] * 9 + [0.25],
                "mlp_hidden": 992, "value_bins": 128}


def geometry(settings: dict) -> dict:
    """The shapes ChessTransformer(**settings) builds (model/model.py:38-53,178-199)."""
    d = settings.get("d_model", 128)
    layers = settings.get("num_layers", 4)
    heads = settings.get("n_heads", 4)
    ratio = settings.get("qk_ratio", 1.0)
    ratios = list(ratio) if isinstance(ratio, (list, tuple)) else [ratio] * layers
    d_head = d // heads
    hidden = settings.get("mlp_hidden") or max(32, int(8 / 3 * d) // 32 * 32)
    return {"d": d, "layers": layers, "heads": heads, "kv_heads": settings.get("kv_heads") or heads, "dv": d_head,
            "dqs": [max(1, round(r * d_head)) for r in ratios], "hidden": hidden, "templates": settings.get("position_templates", 8),
            "bins": settings.get("value_bins", 128)}


def hadamard(size: int) -> torch.Tensor:
    """Sylvester's +-1 Hadamard matrix (model/int8_blocks.py:54-58)."""
    matrix = torch.ones(1, 1)
    while matrix.shape[0] < size:
        matrix = torch.cat([torch.cat([matrix, matrix], 1), torch.cat([matrix, -matrix], 1)], 0)
    return matrix


FP16_LAST_LAYERS = 1  # engine/quantization.py:46: the blocks at the end that stay fp16


def down_inputs(hidden: int) -> int:
    return -(-hidden // DOWN_INPUT_MULTIPLE) * DOWN_INPUT_MULTIPLE


def round_to_nearest(weight: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Symmetric int8 rows, scale = absmax / 127: GPTQ (engine/quantization.py:76-99) with a diagonal Hessian."""
    weight = weight.double()
    scale = weight.abs().amax(dim=1).clamp(min=1e-20) / INT8_MAX
    return (weight / scale[:, None]).round().clamp(-INT8_MAX, INT8_MAX).to(torch.int8), scale.float()


def quantize(state: dict, settings: dict, layers: list[int] | None = None) -> dict:
    """Int8Weights of a state dict, laid out as engine/quantization.py:129-139 lays them out (projection = Q|K|V|template
    mix rows, gate_up = gate rows then up rows, down zero-padded to a multiple of 128 inputs and rotated by the
    block-diagonal Hadamard matrix / 32), rounded to nearest."""
    g = geometry(settings)
    weights = {}
    for i in (range(g["layers"]) if layers is None else layers):
        p = f"encoder.{i}."
        projection = torch.cat([state[p + n + ".weight"].double() for n in ("Q", "K", "V", "template_mix")])
        gate_up = torch.cat([state[p + "mlp.gate_projection.weight"].double(), state[p + "mlp.up_projection.weight"].double()])
        width = down_inputs(g["hidden"])
        rotation = torch.block_diag(*[hadamard(HADAMARD_BLOCK)] * (width // HADAMARD_BLOCK)).double()
        down = nn.functional.pad(state[p + "mlp.down_projection.weight"].double().cpu(), (0, width - g["hidden"])) @ rotation / HADAMARD_BLOCK
        weights[i] = {"projection": round_to_nearest(projection), "gate_up": round_to_nearest(gate_up), "down": round_to_nearest(down)}
    return weights


def synthetic_state_dict(settings: dict, seed: int, std: float = 0.02) -> dict[str, torch.Tensor]:
    """Random-init fp32 weights of a network with these settings (the benchmark configs' N(0, 0.02)), named as the
    reference's ChessTransformer.state_dict() names them. Gains 1, the input skip's scales 0.8 and 0.5."""
    g = geometry(settings)
    d, H, KV, dv, P = g["d"], g["heads"], g["kv_heads"], g["dv"], g["templates"]
    generator = torch.Generator().manual_seed(seed)
    normal = lambda *shape: std * torch.randn(*shape, generator=generator)
    state = {"embed.weight": torch.randn(BOARD_VOCAB_SIZE, d, generator=generator), "position_embed": torch.randn(TOKENS_PER_BOARD, d, generator=generator),
             "square_features.table": normal(FEATURE_TABLE_ROWS, d), "templates": normal(P, 64, 64), "ln.weight": torch.ones(d)}
    for i, dq in enumerate(g["dqs"]):
        p = f"encoder.{i}."
        state.update({p + "Q.weight": normal(H * dq, d), p + "Q.bias": normal(H * dq), p + "K.weight": normal(KV * dq, d),
                      p + "K.bias": normal(KV * dq), p + "V.weight": normal(KV * dv, d), p + "V.bias": normal(KV * dv),
                      p + "q_norm.weight": torch.ones(dq), p + "k_norm.weight": torch.ones(dq), p + "ln1.weight": torch.ones(d),
                      p + "ln2.weight": torch.ones(d), p + "combine_heads.weight": normal(d, d), p + "combine_heads.bias": normal(d),
                      p + "mlp.up_projection.weight": normal(g["hidden"], d), p + "mlp.gate_projection.weight": normal(g["hidden"], d),
                      p + "mlp.down_projection.weight": normal(d, g["hidden"]), p + "template_mix.weight": normal(P * H, d),
                      p + "template_mix.bias": normal(P * H), p + "residual_scale": torch.full((1,), 0.8),
                      p + "input_scale": torch.full((1,), 0.5)})
    state.update({"board_down_project.0.weight": normal(VALUE_TOKEN_DIM, d), "board_down_project.0.bias": normal(VALUE_TOKEN_DIM),
                  "eval_head.0.weight": normal(d, TOKENS_PER_BOARD * VALUE_TOKEN_DIM), "eval_head.0.bias": normal(d),
                  "eval_head.2.weight": normal(g["bins"], d), "eval_head.2.bias": normal(g["bins"]),
                  "from_projection.weight": normal(d, d), "from_projection.bias": normal(d), "to_projection.weight": normal(d, d),
                  "to_projection.bias": normal(d), "promotion_projection.weight": normal(4, d), "promotion_projection.bias": normal(4)})
    return state


def _pointer(tensor: torch.Tensor) -> int:
    return tensor.data_ptr()


class Int8Network(nn.Module):
    """Fry's network on one GPU, its blocks int8 where `weights` has them and fp16 otherwise (the reference's int8_model
    layout). forward(boards [B, 70] int64 cuda) -> rows [B, 1969] fp32."""

    def __init__(self, state: dict, settings: dict, weights: dict, device: torch.device | str | None = None):
        super().__init__()
        device = torch.device(device if device is not None else "cuda")
        if device.type != "cuda":
            raise FryError("Int8Network runs on a CUDA device only")
        if device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        g = geometry(settings)
        # the blocks without int8 weights run in fp16, as the reference's quantize_blocks keeps them (FusedBlock,
        # model/int8_blocks.py:292-298): the engine's layout keeps the last block and ENGINE_FP16_BLOCKS more in fp16
        self.settings, self.geometry, self.d_model, self.eps = settings, g, g["d"], EPS
        s = FP16_RESIDUAL_SCALE
        half = lambda t: t.detach().to(device=device, dtype=torch.float16).contiguous()
        single = lambda t: t.detach().to(device=device, dtype=torch.float32).contiguous()
        self.tensors = {"embed": half(state["embed.weight"].float() * s), "position": half(state["position_embed"].float() * s),
                        "table": half(state["square_features.table"].float() * s), "templates": half(state["templates"]),
                        "ln": half(state["ln.weight"])}
        self.blocks = []
        for i, dq in enumerate(g["dqs"]):
            p = f"encoder.{i}."
            block = {"ln1": half(state[p + "ln1.weight"]), "ln2": half(state[p + "ln2.weight"]),
                     "residual_scale": half(state[p + "residual_scale"]), "input_scale": half(state[p + "input_scale"]),
                     "q_gain": half(state[p + "q_norm.weight"]), "k_gain": half(state[p + "k_norm.weight"]),
                     "projection_bias": half(torch.cat([state[p + n + ".bias"] for n in ("Q", "K", "V", "template_mix")])),
                     "combine_heads": half(state[p + "combine_heads.weight"].float() * s),
                     "combine_heads_bias": half(state[p + "combine_heads.bias"].float() * s)}
            if i in weights:
                w = weights[i]
                width = w["down"][0].shape[1]
                if width != down_inputs(g["hidden"]):
                    raise FryError(f"block {i}'s down takes {width} inputs, not the padded hidden width {down_inputs(g['hidden'])}")
                block.update({"precision": BLOCK_INT8, "projection": w["projection"][0].to(device).contiguous(),
                              "projection_scale": single(w["projection"][1]), "gate_up": w["gate_up"][0].to(device).contiguous(),
                              "gate_up_scale": single(w["gate_up"][1]), "down": w["down"][0].to(device).contiguous(),
                              "down_scale": single(w["down"][1].float() * s)})
            else:
                # FusedBlock's weights in nn.Linear's [out, in] layout (the reference keeps them transposed), the down
                # scaled into the stream's 1/16 before the fp16 rounding as scale_residual_stream does (model/model.py:235-243)
                block.update({"precision": BLOCK_FP16,
                              "projection": half(torch.cat([state[p + n + ".weight"] for n in ("Q", "K", "V", "template_mix")])),
                              "gate_up": half(torch.cat([state[p + "mlp.gate_projection.weight"], state[p + "mlp.up_projection.weight"]])),
                              "down": half(state[p + "mlp.down_projection.weight"].float() * s)})
            self.blocks.append(block)
        # heads (model/fused_blocks.py:815-824), folded in fp64
        from_w, from_b = state["from_projection.weight"].double(), state["from_projection.bias"].double()
        to_w, to_b = state["to_projection.weight"].double(), state["to_projection.bias"].double()
        scale = 1 / math.sqrt(g["d"])
        self.tensors.update({
            "a_weight": half(to_w.T @ from_w * scale),   # row n = column n of A = W_f^T W_t / sqrt d
            "a_bias": single(to_w.T @ from_b * scale),
            "narrow_weight": single(torch.cat([(to_b @ from_w)[None] * scale, state["promotion_projection.weight"].double(),
                                               state["board_down_project.0.weight"].double()])),
            "narrow_bias": single(torch.cat([(from_b @ to_b)[None] * scale, state["promotion_projection.bias"].double(),
                                             state["board_down_project.0.bias"].double()])),
            "hidden_weight": single(state["eval_head.0.weight"]), "hidden_bias": single(state["eval_head.0.bias"]),
            "out_weight": single(state["eval_head.2.weight"]), "out_bias": single(state["eval_head.2.bias"])})
        self.device = device
        with torch.cuda.device(device):
            self.tensors["templates"] = pair_templates(self.tensors["templates"])
            torch.cuda.current_stream(device).synchronize()
        self._network = self._struct()
        self._handle = next(_HANDLES)
        _NETWORKS[self._handle] = weakref.ref(self)
        weakref.finalize(self, _NETWORKS.pop, self._handle, None)

    def _struct(self) -> FryNetwork:
        g, t = self.geometry, self.tensors
        blocks = (FryBlock * len(self.blocks))()
        for i, (dq, b) in enumerate(zip(g["dqs"], self.blocks)):
            pointer = lambda name: _pointer(b[name]) if name in b else None
            blocks[i] = FryBlock(dq, *(pointer(name) for name in ("ln1", "ln2", "residual_scale", "input_scale", "q_gain", "k_gain",
                                                                  "projection", "projection_scale", "projection_bias", "combine_heads",
                                                                  "combine_heads_bias", "gate_up", "gate_up_scale", "down", "down_scale")),
                                 b["precision"])
        self._blocks_array = blocks
        return FryNetwork(g["d"], g["layers"], g["heads"], g["kv_heads"], g["dv"], g["templates"], g["hidden"], down_inputs(g["hidden"]),
                          self.eps, _pointer(t["embed"]), _pointer(t["position"]), _pointer(t["table"]), _pointer(t["templates"]),
                          ctypes.cast(blocks, ctypes.POINTER(FryBlock)),
                          heads_struct(t["ln"], t["a_weight"], t["a_bias"], t["narrow_weight"], t["narrow_bias"], t["hidden_weight"],
                                       t["hidden_bias"], t["out_weight"], t["out_bias"]))

    def forward_lean(self, lean_rows: torch.Tensor) -> torch.Tensor:
        """Lean lanes' rows uint8 [B, LEAN_ROW] cuda (tokens, then int16 answer columns) -> answers fp32 [B, LEAN_COLUMNS]:
        forward(tokens) gathered at the columns (engine/inference.py:130-135), the gather in the heads' last kernel. Runs
        as the torch op fry::forward_lean."""
        if not lean_rows.is_cuda or lean_rows.device != self.device:
            raise FryError(f"Int8Network on {self.device} got lean rows on {lean_rows.device}")
        return torch.ops.fry.forward_lean(lean_rows, self._handle)

    def workspace_bytes(self, boards: int) -> int:
        return library().fry_forward_workspace_bytes(ctypes.byref(self._network), boards)

    def forward(self, board_state: torch.Tensor) -> torch.Tensor:
        """boards [B, 70] tokens on this network's device -> answer rows fp32 [B, 1969], as the torch op fry::forward, so
        torch.compile sees the forward through the op's fake implementation, as it sees the reference's custom ops."""
        if not board_state.is_cuda or board_state.device != self.device:
            raise FryError(f"Int8Network on {self.device} got boards on {board_state.device}")
        return torch.ops.fry.forward(board_state.to(torch.int64), self._handle)

    def _rows(self, boards: torch.Tensor) -> torch.Tensor:
        boards = boards.contiguous()
        if boards.dtype != torch.int64 or boards.dim() != 2 or boards.shape[1] != TOKENS_PER_BOARD:
            raise FryError(f"boards are int64 [B, {TOKENS_PER_BOARD}] tokens, got {boards.dtype} {tuple(boards.shape)}")
        B = boards.shape[0]
        rows = torch.empty(B, ANSWER_WIDTH, device=self.device, dtype=torch.float32)
        lib = library()
        size = lib.fry_forward_workspace_bytes(ctypes.byref(self._network), B)
        workspace = torch.empty(max(size, 1), device=self.device, dtype=torch.uint8)
        lib.fry_forward(ctypes.byref(self._network), ctypes.c_void_p(boards.data_ptr()), B, ctypes.c_void_p(rows.data_ptr()),
                        ctypes.c_void_p(workspace.data_ptr()), size, ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream))
        return rows

    def _lean_answers(self, lean_rows: torch.Tensor) -> torch.Tensor:
        lean_rows = lean_rows.contiguous()
        if lean_rows.dtype != torch.uint8 or lean_rows.dim() != 2 or lean_rows.shape[1] != LEAN_ROW:
            raise FryError(f"lean rows are uint8 [B, {LEAN_ROW}], got {lean_rows.dtype} {tuple(lean_rows.shape)}")
        B = lean_rows.shape[0]
        answers = torch.empty(B, LEAN_COLUMNS, device=self.device, dtype=torch.float32)
        lib = library()
        size = lib.fry_forward_lean_workspace_bytes(ctypes.byref(self._network), B)
        workspace = torch.empty(max(size, 1), device=self.device, dtype=torch.uint8)
        lib.fry_forward_lean(ctypes.byref(self._network), ctypes.c_void_p(lean_rows.data_ptr()), B, ctypes.c_void_p(answers.data_ptr()),
                             ctypes.c_void_p(workspace.data_ptr()), size, ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream))
        return answers


# The networks the ops below run, by handle: an op takes tensors and plain values, so a network is named by an integer
# that Int8Network sets up (torch.compile keeps it as a constant of the traced graph). The registry holds weak
# references: a network that is gone is refused, not kept alive.
_NETWORKS: dict[int, "weakref.ReferenceType[Int8Network]"] = {}
_HANDLES = itertools.count(1)


def _registered(handle: int) -> Int8Network:
    found = _NETWORKS.get(handle)
    network = found() if found is not None else None
    if network is None:
        raise FryError(f"no live Int8Network has handle {handle}")
    return network


@torch.library.custom_op("fry::forward", mutates_args=())
def forward_op(boards: torch.Tensor, network: int) -> torch.Tensor:
    """`FusedTransformer.forward` + `answer_rows` (model/fused_blocks.py:856-862, engine/inference.py:19-23) of the
    network with this handle: boards int64 [B, 70] -> rows fp32 [B, 1969], one fry_forward on the current stream."""
    return _registered(network)._rows(boards)


@forward_op.register_fake
def _(boards, network):
    return boards.new_empty(boards.shape[0], ANSWER_WIDTH, dtype=torch.float32)


@torch.library.custom_op("fry::forward_lean", mutates_args=())
def forward_lean_op(lean_rows: torch.Tensor, network: int) -> torch.Tensor:
    """The lean lanes' forward (engine/inference.py:130-135) of the network with this handle: rows uint8 [B, 508] ->
    answers fp32 [B, 219], one fry_forward_lean on the current stream."""
    return _registered(network)._lean_answers(lean_rows)


@forward_lean_op.register_fake
def _(lean_rows, network):
    return lean_rows.new_empty(lean_rows.shape[0], LEAN_COLUMNS, dtype=torch.float32)


def load_checkpoint(checkpoint_path: Path) -> tuple[dict, dict]:
    """(state_dict, model_settings) of a checkpoint written by the reference's save_checkpoint (model/checkpoint.py:22-38)."""
    checkpoint = torch.load(checkpoint_path, map_location="cpu", weights_only=False)
    settings = dict(checkpoint["model_settings"])
    if settings.pop("loops", 1) != 1:
        raise FryError(f"{checkpoint_path} runs its blocks more than once, which the network here cannot")
    return {name: tensor.float() if tensor.is_floating_point() else tensor for name, tensor in checkpoint["state_dict"].items()}, settings


def int8_model(checkpoint_path: Path, fp16_blocks: int = 0, weights: dict | None = None, device: torch.device | str | None = None,
               calibration: tuple[torch.Tensor, torch.Tensor | None] | None = None) -> Int8Network:
    """`engine.inference.int8_model` (engine/inference.py:267-272) on this engine: the blocks `weights` has run in int8,
    the others in fp16. `weights` are Int8Weights (the reference's cached GPTQ weights load unchanged, their blocks
    fixing the layout). Without them, as the reference does, the checkpoint's weights come from
    `quantization.int8_weights(checkpoint_path, fp16_blocks, calibration)`: the weights the reference cached for this
    checkpoint, or with `calibration` (boards int64 [n, 70], and for fp16_blocks > 0 their legal moves bool [n, 1968])
    GPTQ over those positions on this GPU with the fp16_blocks blocks of the largest block_errors kept fp16, cached."""
    device = torch.device(device if device is not None else "cuda")
    if device.type != "cuda":
        raise FryError("int8_model runs on a CUDA device only")
    if device.index is None:
        device = torch.device("cuda", torch.cuda.current_device())
    state, settings = load_checkpoint(Path(checkpoint_path))
    if weights is None:
        from .quantization import int8_weights
        weights = int8_weights(Path(checkpoint_path), fp16_blocks, calibration, device)
    return Int8Network(state, settings, weights, device)
