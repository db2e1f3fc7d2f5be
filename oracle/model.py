"""Fry's fp32 network restated on the CPU. TEST INFRASTRUCTURE ONLY.

Follows `model/model.py` of the reference: the square features
(`:102-174`), the transformer block (`:37-99`) and `ChessTransformer.forward`
(`:245-270`), plus `expected_score` (`:23-24`) and `engine/inference.py:19-23`
(`answer_rows`). Parameters are a plain dict named exactly like the
reference's `ChessTransformer.state_dict()`, so one dict loads into both.

This fp32 forward is also the reference's only CPU evaluation of the network
(`engine/inference.py:274-278`, `cpu_batches`), which is what `bench.py`'s
reference arm times.
"""
import math

import numpy as np
import torch
import torch.nn.functional as F

from oracle.encoding import (BOARD_VOCAB_SIZE, MOVE_FROM_SQUARES, MOVE_TO_SQUARES, NUM_MOVE_IDS, NUM_PIECE_CODES, NUM_PIECE_TYPES,
                             NUM_SQUARES, PROMOTION_MOVE_IDS, PROMOTION_PIECES, PROMOTION_TO_SQUARES, TOKENS_PER_BOARD)

VALUE_TOKEN_DIM = 16          # model/model.py:7
VALUE_BINS = 128              # :8
EPS = 1e-5                    # every RMSNorm of the model, :55-60,221

# piece codes and feature geometry, model/model.py:103-116
PAWN, KNIGHT, QUEEN, KING = 1, 2, 5, 6
THEIRS = NUM_PIECE_TYPES
EDGE = NUM_PIECE_CODES
DIRECTIONS = [(0, 1), (0, -1), (1, 0), (-1, 0), (1, 1), (-1, 1), (1, -1), (-1, -1)]
KNIGHT_JUMPS = [(1, 2), (2, 1), (2, -1), (1, -2), (-1, -2), (-2, -1), (-2, 1), (-1, 2)]
NO_PIECE = 15 * 15
OFFSET_ROWS = NO_PIECE + 1
NEIGHBOUR_ROWS = NUM_PIECE_CODES + 1
LINE_ROWS = 1 + 12 * 7
KNIGHT_ROWS = 3 * 3
PAWN_ROWS = 1 + 2 * 7
SLOT_ROWS = [OFFSET_ROWS] * 4 + [NEIGHBOUR_ROWS] * 8 + [LINE_ROWS] * 8 + [KNIGHT_ROWS] + [PAWN_ROWS] * 2
FEATURES = len(SLOT_ROWS)                                  # 23
FEATURE_TABLE_ROWS = sum(SLOT_ROWS)                        # 1735
ROW_OFFSETS = np.concatenate([[0], np.cumsum(SLOT_ROWS)[:-1]]).astype(np.int64)   # model/model.py:134


def _step(square: int, file_step: int, rank_step: int) -> int:
    """model/model.py:118-120: the square a step away, or 64 past the edge."""
    file, rank = square % 8 + file_step, square // 8 + rank_step
    return rank * 8 + file if 0 <= file < 8 and 0 <= rank < 8 else NUM_SQUARES


OFFSETS = np.array([[(s // 8 - p // 8 + 7) * 15 + s % 8 - p % 8 + 7 for p in range(64)] for s in range(64)], dtype=np.int64)  # :139
RAYS = np.array([[[_step(s, d[0] * k, d[1] * k) for k in range(1, 8)] for d in DIRECTIONS] for s in range(64)], dtype=np.int64)  # :142
JUMPS = np.array([[_step(s, *j) for j in KNIGHT_JUMPS] for s in range(64)], dtype=np.int64)                                  # :144


def mlp_hidden_width(d_model: int, mlp_ratio: float | None = None) -> int:
    """model/model.py:11-13."""
    ratio = 8 / 3 if mlp_ratio is None else mlp_ratio
    return max(32, int(ratio * d_model) // 32 * 32)


def geometry(settings: dict) -> dict:
    """The shapes `ChessTransformer(**settings)` builds (model/model.py:178-199, 38-53)."""
    d = settings.get("d_model", 128)
    layers = settings.get("num_layers", 4)
    heads = settings.get("n_heads", 4)
    ratio = settings.get("qk_ratio", 1.0)
    ratios = list(ratio) if isinstance(ratio, (list, tuple)) else [ratio] * layers
    d_head = d // heads
    kv = settings.get("kv_heads") or heads
    hidden = settings.get("mlp_hidden") or mlp_hidden_width(d)
    return {"d": d, "layers": layers, "heads": heads, "kv_heads": kv, "dv": d_head,
            "dqs": [max(1, round(r * d_head)) for r in ratios], "hidden": hidden,
            "templates": settings.get("position_templates", 8), "bins": settings.get("value_bins", VALUE_BINS)}


def parameter_shapes(settings: dict) -> dict[str, tuple[int, ...]]:
    """Every learned tensor of the reference's state_dict with its shape."""
    g = geometry(settings)
    d, H, KV, dv, P = g["d"], g["heads"], g["kv_heads"], g["dv"], g["templates"]
    shapes = {"embed.weight": (BOARD_VOCAB_SIZE, d), "position_embed": (TOKENS_PER_BOARD, d),
              "square_features.table": (FEATURE_TABLE_ROWS, d), "templates": (P, NUM_SQUARES, NUM_SQUARES)}
    for i, dq in enumerate(g["dqs"]):
        p = f"encoder.{i}."
        shapes.update({p + "Q.weight": (H * dq, d), p + "Q.bias": (H * dq,), p + "K.weight": (KV * dq, d), p + "K.bias": (KV * dq,),
                       p + "V.weight": (KV * dv, d), p + "V.bias": (KV * dv,), p + "q_norm.weight": (dq,), p + "k_norm.weight": (dq,),
                       p + "ln1.weight": (d,), p + "ln2.weight": (d,), p + "combine_heads.weight": (d, d), p + "combine_heads.bias": (d,),
                       p + "mlp.up_projection.weight": (g["hidden"], d), p + "mlp.gate_projection.weight": (g["hidden"], d),
                       p + "mlp.down_projection.weight": (d, g["hidden"]), p + "template_mix.weight": (P * H, d),
                       p + "template_mix.bias": (P * H,), p + "residual_scale": (1,), p + "input_scale": (1,)})
    shapes.update({"board_down_project.0.weight": (VALUE_TOKEN_DIM, d), "board_down_project.0.bias": (VALUE_TOKEN_DIM,),
                   "eval_head.0.weight": (d, TOKENS_PER_BOARD * VALUE_TOKEN_DIM), "eval_head.0.bias": (d,),
                   "eval_head.2.weight": (g["bins"], d), "eval_head.2.bias": (g["bins"],),
                   "from_projection.weight": (d, d), "from_projection.bias": (d,), "to_projection.weight": (d, d), "to_projection.bias": (d,),
                   "promotion_projection.weight": (4, d), "promotion_projection.bias": (4,), "ln.weight": (d,)})
    return shapes


def move_buffers() -> dict[str, torch.Tensor]:
    """The persistent move buffers of ChessTransformer (model/model.py:209-215)."""
    return {"from_squares": torch.from_numpy(MOVE_FROM_SQUARES), "to_squares": torch.from_numpy(MOVE_TO_SQUARES),
            "promotion_move_ids": torch.from_numpy(PROMOTION_MOVE_IDS), "promotion_to_squares": torch.from_numpy(PROMOTION_TO_SQUARES),
            "promotion_pieces": torch.from_numpy(PROMOTION_PIECES)}


def seeded_state_dict(settings: dict, seed: int, *, std: float = 0.02, template_std: float = 0.5, table_std: float = 0.1,
                      gain_jitter: float = 0.1, from_scale: float = 1.0) -> dict[str, torch.Tensor]:
    """Synthetic fp32 weights for a network of these settings, drawn in sorted-name order from one seeded generator.

    Random-init N(0, std) weights as the benchmark configs describe; the templates and the square-feature table are
    drawn wider because zeros there would hide a missing bias or feature (the reference's tests randomise them the same
    way, tests/test_int8.py:316-318). RMSNorm gains are 1 + N(0, gain_jitter), the input skip's scales 0.8 and 0.5
    (tests/test_model.py:20-25).
    """
    generator = torch.Generator().manual_seed(seed)
    state = {}
    for name, shape in sorted(parameter_shapes(settings).items()):
        if name.endswith("residual_scale"):
            state[name] = torch.full(shape, 0.8)
        elif name.endswith("input_scale"):
            state[name] = torch.full(shape, 0.5)
        elif name.endswith("norm.weight") or name.endswith("ln1.weight") or name.endswith("ln2.weight") or name == "ln.weight":
            state[name] = 1 + gain_jitter * torch.randn(shape, generator=generator)
        elif name == "templates":
            state[name] = template_std * torch.randn(shape, generator=generator)
        elif name == "square_features.table":
            state[name] = table_std * torch.randn(shape, generator=generator)
        elif name == "position_embed" or name == "embed.weight":
            state[name] = torch.randn(shape, generator=generator)
        else:
            state[name] = std * torch.randn(shape, generator=generator)
    state["from_projection.weight"] = state["from_projection.weight"] * from_scale
    state.update(move_buffers())
    return state


def square_feature_indices(boards: torch.Tensor) -> torch.Tensor:
    """B x 64 x 23: each square's row within each feature's rows, `SquareFeatures.indices` (model/model.py:147-169)."""
    boards = boards.long()
    squares = boards[:, :NUM_SQUARES]
    padded = F.pad(squares, (0, 1), value=EDGE)
    offsets_table = torch.from_numpy(OFFSETS)
    offsets = []
    for code in (KING, KING + THEIRS, QUEEN, QUEEN + THEIRS):
        present = squares == code
        square = present.int().argmax(dim=1)
        offsets.append(torch.where(present.any(dim=1, keepdim=True), offsets_table[:, square].T, NO_PIECE))

    def first_along(along, found):
        distance = found.int().argmax(dim=-1, keepdim=True)
        code = torch.where(found.any(dim=-1, keepdim=True), along.gather(-1, distance), 0)
        return code.squeeze(-1), distance.squeeze(-1)

    along = padded[:, torch.from_numpy(RAYS)]
    first, distance = first_along(along, (along != 0) & (along != EDGE))
    lines = torch.where(first > 0, 1 + (first - 1) * 7 + distance, 0)
    jumps = padded[:, torch.from_numpy(JUMPS)]
    knights = (jumps == KNIGHT).sum(dim=-1).clamp(max=2) * 3 + (jumps == KNIGHT + THEIRS).sum(dim=-1).clamp(max=2)
    file = along[:, :, :2]
    pawn, pawn_distance = first_along(file, (file == PAWN) | (file == PAWN + THEIRS))
    pawns = torch.where(pawn > 0, 1 + (pawn == PAWN + THEIRS).long() * 7 + pawn_distance, 0)
    return torch.cat([torch.stack(offsets, dim=-1), along[..., 0], lines, knights.unsqueeze(-1), pawns], dim=-1)


def square_features(state: dict, boards: torch.Tensor) -> torch.Tensor:
    """B x 64 x d, the 23 table rows summed (model/model.py:171-174)."""
    rows = square_feature_indices(boards) + torch.from_numpy(ROW_OFFSETS)
    return state["square_features.table"][rows].sum(dim=-2)


def _linear(state: dict, name: str, x: torch.Tensor) -> torch.Tensor:
    bias = state.get(name + ".bias")
    return F.linear(x, state[name + ".weight"], bias)


def block_forward(state: dict, g: dict, i: int, x: torch.Tensor, templates: torch.Tensor, original: torch.Tensor) -> torch.Tensor:
    """`TransformerBlock.forward` (model/model.py:71-99)."""
    p = f"encoder.{i}."
    B, T, d = x.shape
    H, KV, dq, dv = g["heads"], g["kv_heads"], g["dqs"][i], g["dv"]
    residual = state[p + "residual_scale"] * x + state[p + "input_scale"] * original
    x_norm = F.rms_norm(residual, (d,), state[p + "ln1.weight"], EPS)
    q = F.rms_norm(_linear(state, p + "Q", x_norm).reshape(B, T, H, dq), (dq,), state[p + "q_norm.weight"], EPS).transpose(1, 2)
    k = F.rms_norm(_linear(state, p + "K", x_norm).reshape(B, T, KV, dq), (dq,), state[p + "k_norm.weight"], EPS).transpose(1, 2)
    v = _linear(state, p + "V", x_norm).reshape(B, T, KV, dv).transpose(1, 2)
    k = k.repeat_interleave(H // KV, dim=1)
    v = v.repeat_interleave(H // KV, dim=1)
    scores = (q @ k.transpose(-2, -1)) / math.sqrt(dq)
    coefficients = _linear(state, p + "template_mix", x_norm[:, :NUM_SQUARES]).reshape(B, NUM_SQUARES, H, g["templates"])
    bias = torch.einsum("biht,tij->bhij", coefficients, templates)
    scores = scores + F.pad(bias, (0, T - NUM_SQUARES, 0, T - NUM_SQUARES))
    attended = (torch.softmax(scores, dim=-1) @ v).transpose(1, 2).reshape(B, T, d)
    residual = residual + _linear(state, p + "combine_heads", attended)
    normed = F.rms_norm(residual, (d,), state[p + "ln2.weight"], EPS)
    hidden = F.silu(F.linear(normed, state[p + "mlp.gate_projection.weight"])) * F.linear(normed, state[p + "mlp.up_projection.weight"])
    return residual + F.linear(hidden, state[p + "mlp.down_projection.weight"])


def fp32_forward(state: dict, settings: dict, boards: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """`ChessTransformer.forward` (model/model.py:245-270): move logits [B, 1968] and value logits [B, bins]."""
    g = geometry(settings)
    boards = boards.long()
    B = boards.shape[0]
    embed = (state["embed.weight"][boards] + state["position_embed"]
             + F.pad(square_features(state, boards), (0, 0, 0, TOKENS_PER_BOARD - NUM_SQUARES)))
    x = embed
    for i in range(g["layers"]):
        x = block_forward(state, g, i, x, state["templates"], embed)
    out = F.rms_norm(x, (g["d"],), state["ln.weight"], EPS)
    squares = out[:, :NUM_SQUARES]
    from_vector = _linear(state, "from_projection", squares)
    to_vector = _linear(state, "to_projection", squares)
    promotion = _linear(state, "promotion_projection", squares)
    logits = (from_vector @ to_vector.transpose(1, 2)) / math.sqrt(g["d"])
    combined = logits[:, torch.from_numpy(MOVE_FROM_SQUARES), torch.from_numpy(MOVE_TO_SQUARES)]
    combined[:, torch.from_numpy(PROMOTION_MOVE_IDS)] += promotion[:, torch.from_numpy(PROMOTION_TO_SQUARES), torch.from_numpy(PROMOTION_PIECES)]
    compressed = F.gelu(_linear(state, "board_down_project.0", out)).reshape(B, -1)
    value = _linear(state, "eval_head.2", F.gelu(_linear(state, "eval_head.0", compressed)))
    return combined, value


def value_bin_centres(bins: int) -> torch.Tensor:
    """model/model.py:15-20."""
    edges = torch.linspace(0, 1, bins + 1)
    return (edges[:-1] + edges[1:]) / 2


def expected_score(value_logits: torch.Tensor) -> torch.Tensor:
    """model/model.py:23-24: the bins' softmax times their centres."""
    return torch.softmax(value_logits.float(), dim=-1) @ value_bin_centres(value_logits.shape[-1])


def answer_rows(outputs) -> torch.Tensor:
    """engine/inference.py:19-23: [logits ‖ expected score] per board."""
    if isinstance(outputs, torch.Tensor):
        return outputs
    logits, values = outputs
    return torch.cat([logits.float(), expected_score(values).unsqueeze(1)], dim=1)


assert NUM_MOVE_IDS == 1968
