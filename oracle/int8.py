"""The reference's int8 inference path restated on the CPU. TEST INFRASTRUCTURE ONLY.

The reference computes this path only on the GPU (Triton kernels and NVRTC
CUDA). This module restates each kernel's arithmetic, with the same rounding
points, in torch on the CPU:

- weight layout and rounding: `engine/quantization.py:76-99,124-140`
  (round-to-nearest, which is GPTQ with a diagonal Hessian, tests/test_int8.py:35-41);
- fp16 inference set-up: `engine/inference.py:238-249` (stream scaled by 1/16,
  everything but the heads in fp16) and `model/int8_blocks.py:254-272`;
- `norm_quant` / `mix_norm_quant`: `model/int8_blocks.py:156-175`;
- int8 matmul epilogues: `model/int8_cuda.py:146-182` (the op order the
  reference's CUDA and Triton kernels share), `model/fused_blocks.py:208-225`;
- `rotate_quant`: `model/int8_blocks.py:216-231`;
- template attention: `model/fused_blocks.py:35-97`;
- `combine_heads` linear: `model/fused_blocks.py:229-278` (accumulated in fp32
  here; the reference accumulates in fp16, which only this oracle's tolerance
  covers);
- input embedding: `model/fused_blocks.py:370-393`;
- the B200 head path: `model/fused_blocks.py:815-824,863-874`;
- the block: `model/int8_blocks.py:274-288`, linking `model/fused_blocks.py:357-363`.

int32 sums are exact (fp64 accumulation of int8 products is exact). fp32
steps use IEEE round-to-nearest; an fp32 fused multiply-add is emulated as an
fp64 product-plus-sum rounded once to fp32.
"""
import math

import torch
import torch.nn.functional as F

from oracle.encoding import (MOVE_FROM_SQUARES, MOVE_TO_SQUARES, NUM_SQUARES, PROMOTION_MOVE_IDS, PROMOTION_PIECES, PROMOTION_TO_SQUARES,
                             TOKENS_PER_BOARD)
from oracle.model import EPS, ROW_OFFSETS, geometry, square_feature_indices, value_bin_centres

HADAMARD_BLOCK = 32            # model/int8_blocks.py:15
DOWN_INPUT_MULTIPLE = 128      # :17
INT8_MAX = 127                 # engine/quantization.py:47
FP16_RESIDUAL_SCALE = 1 / 16   # engine/inference.py:239
LOG2E = 1.4426950408889634


def hadamard(size: int) -> torch.Tensor:
    """Sylvester's +-1 Hadamard matrix (model/int8_blocks.py:54-58)."""
    matrix = torch.ones(1, 1)
    while matrix.shape[0] < size:
        matrix = torch.cat([torch.cat([matrix, matrix], 1), torch.cat([matrix, -matrix], 1)], 0)
    return matrix


def down_inputs(hidden: int) -> int:
    """model/int8_blocks.py:61-62."""
    return -(-hidden // DOWN_INPUT_MULTIPLE) * DOWN_INPUT_MULTIPLE


def round_to_nearest(weight: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """(int8 [N, K], fp32 [N]) symmetric per output row: engine/quantization.py:87,94 without error feedback."""
    weight = weight.double()
    scale = weight.abs().amax(dim=1).clamp(min=1e-20) / INT8_MAX
    integers = (weight / scale[:, None]).round().clamp(-INT8_MAX, INT8_MAX)
    return integers.to(torch.int8), scale.float()


def int8_weights(state: dict, settings: dict, layers: list[int] | None = None) -> dict:
    """`Int8Weights` for the given layers (default: all), laid out as engine/quantization.py:129-139 lays them out:
    projection = Q|K|V|template_mix rows, gate_up = gate rows then up rows, down padded to a multiple of 128 inputs
    and rotated by the block-diagonal Hadamard matrix / 32."""
    g = geometry(settings)
    layers = list(range(g["layers"])) if layers is None else layers
    weights = {}
    for i in layers:
        p = f"encoder.{i}."
        projection = torch.cat([state[p + n + ".weight"] for n in ("Q", "K", "V", "template_mix")]).double()
        gate_up = torch.cat([state[p + "mlp.gate_projection.weight"], state[p + "mlp.up_projection.weight"]]).double()
        hidden = g["hidden"]
        width = down_inputs(hidden)
        rotation = torch.block_diag(*[hadamard(HADAMARD_BLOCK)] * (width // HADAMARD_BLOCK)).double()
        down = F.pad(state[p + "mlp.down_projection.weight"].double(), (0, width - hidden)) @ rotation / HADAMARD_BLOCK
        weights[i] = {"projection": round_to_nearest(projection), "gate_up": round_to_nearest(gate_up), "down": round_to_nearest(down)}
    return weights


def fma32(a: torch.Tensor, b: torch.Tensor, c: torch.Tensor) -> torch.Tensor:
    return (a.double() * b.double() + c.double()).float()


def rint(x: torch.Tensor) -> torch.Tensor:
    """Round half to even, as libdevice.rint and cvt.rni do."""
    return torch.round(x)


def norm_quant(x: torch.Tensor, gain: torch.Tensor, eps: float = EPS) -> tuple[torch.Tensor, torch.Tensor]:
    """model/int8_blocks.py:156-175 (MIX off): RMSNorm with gain in fp32, then int8 rows, a row's scale absmax / 127."""
    xf = x.float()
    D = xf.shape[-1]
    inverse = torch.rsqrt((xf.double() * xf.double()).sum(-1) / D + eps).float()
    y = xf * inverse[..., None] * gain.float()
    absmax = y.abs().amax(-1).clamp(min=1e-20)
    q = rint(y * (127.0 / absmax)[..., None]).to(torch.int8)
    return q, absmax / 127.0


def mix(x: torch.Tensor, original: torch.Tensor, residual_scale: torch.Tensor, input_scale: torch.Tensor) -> torch.Tensor:
    """model/int8_blocks.py:166-170: fp16(rs * x + is * original), as fma(rs, x, is * original)."""
    return fma32(residual_scale.float(), x.float(), input_scale.float() * original.float()).half()


def int8_matmul(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """Exact int32 sums x[M, K] . w[N, K]^T (fp64 holds every partial sum of int8 products exactly)."""
    return (x.double() @ w.double().T).to(torch.int32)


def epilogue_bias(acc, x_scale, w_scale, bias) -> torch.Tensor:
    """EPI 0, model/int8_cuda.py:163-165: fp16(fma(acc * xs, ws, bias))."""
    value = acc.float() * x_scale.float()[:, None]
    return fma32(value, w_scale.float()[None, :], bias.float()[None, :]).half()


def epilogue_gated(acc_gate, acc_up, x_scale, w_scale_gate, w_scale_up) -> torch.Tensor:
    """EPI 1, model/int8_cuda.py:166-170: fp16((g * sigmoid(g)) * u), g and u dequantised as (acc * xs) * ws."""
    xs = x_scale.float()[:, None]
    gate = (acc_gate.float() * xs) * w_scale_gate.float()[None, :]
    up = (acc_up.float() * xs) * w_scale_up.float()[None, :]
    sigmoid = torch.sigmoid(gate.double()).float()
    return ((gate * sigmoid) * up).half()


def epilogue_residual(acc, x_scale, w_scale, residual) -> torch.Tensor:
    """EPI 2, model/int8_cuda.py:171-172: fp16(fma(acc * xs, ws, residual))."""
    value = acc.float() * x_scale.float()[:, None]
    return fma32(value, w_scale.float()[None, :], residual.float()).half()


def epilogue_mixing(acc, x_scale, w_scale, residual, original, residual_scale, input_scale) -> torch.Tensor:
    """EPI 3, model/int8_cuda.py:171-176: the stream rounded to fp16, then the next block's input mix."""
    value = acc.float() * x_scale.float()[:, None]
    stream = fma32(value, w_scale.float()[None, :], residual.float()).half().float()
    return fma32(stream, residual_scale.float(), original.float() * input_scale.float()).half()


def int8_linear(x, x_scale, weight, weight_scale, bias=None, residual=None, gated=False, original=None,
                residual_scale=None, input_scale=None) -> torch.Tensor:
    """The op `chess::int8_linear` (model/int8_blocks.py:132-139) on 2-D operands: x [M, K] int8, weight [N, K] int8."""
    if gated:
        n = weight.shape[0] // 2
        acc = int8_matmul(x, weight)
        return epilogue_gated(acc[:, :n], acc[:, n:], x_scale, weight_scale[:n], weight_scale[n:])
    acc = int8_matmul(x, weight)
    if residual is None:
        return epilogue_bias(acc, x_scale, weight_scale, bias)
    if original is None:
        return epilogue_residual(acc, x_scale, weight_scale, residual)
    return epilogue_mixing(acc, x_scale, weight_scale, residual, original, residual_scale, input_scale)


def rotate_quant(h: torch.Tensor, width: int) -> tuple[torch.Tensor, torch.Tensor]:
    """model/int8_blocks.py:216-231: h [M, hidden] fp16 zero-padded to width, times blockdiag(H32), int8 rows."""
    padded = F.pad(h.double(), (0, width - h.shape[-1]))
    blocks = padded.reshape(*padded.shape[:-1], width // HADAMARD_BLOCK, HADAMARD_BLOCK)
    rotated = (blocks @ hadamard(HADAMARD_BLOCK).double()).reshape(padded.shape).float()
    absmax = rotated.abs().amax(-1).clamp(min=1e-20)
    q = rint(rotated * (127.0 / absmax)[..., None]).to(torch.int8)
    return q, absmax / 127.0


def template_attention(projected: torch.Tensor, templates: torch.Tensor, q_gain: torch.Tensor, k_gain: torch.Tensor, heads: int,
                       kv_heads: int, dq: int, dv: int, templates_count: int, eps: float = EPS) -> torch.Tensor:
    """model/fused_blocks.py:35-97 with its rounding points: q and k normalised and rounded to fp16, the template bias
    rounded to fp16, scores and softmax in fp32, probabilities rounded to fp16 for the value product, the sum divided
    by the unrounded total. projected [B, 70, heads*dq + kv*dq + kv*dv + heads*templates] fp16 -> [B, 70, heads*dv]."""
    B, T, _ = projected.shape
    q, k, v, c = projected.double().split([heads * dq, kv_heads * dq, kv_heads * dv, heads * templates_count], dim=-1)
    group = heads // kv_heads

    def normed(t, n, gain):
        t = t.reshape(B, T, n, dq)
        inverse = torch.rsqrt((t * t).sum(-1, keepdim=True) / dq + eps).float().double()
        return (t * inverse * gain.double()).float().half().double()

    qn = normed(q, heads, q_gain).transpose(1, 2)                                      # B H T dq
    kn = normed(k, kv_heads, k_gain).transpose(1, 2).repeat_interleave(group, 1)
    vv = v.reshape(B, T, kv_heads, dv).transpose(1, 2).repeat_interleave(group, 1)
    scale = torch.tensor(1 / math.sqrt(dq), dtype=torch.float32).double()
    scores = ((qn @ kn.transpose(-2, -1)).float().double() * scale).float()
    coefficients = c[:, :NUM_SQUARES].reshape(B, NUM_SQUARES, heads, templates_count)
    bias = torch.einsum("biht,tij->bhij", coefficients, templates.double()).float().half().float()
    scores = scores + F.pad(bias, (0, T - NUM_SQUARES, 0, T - NUM_SQUARES))
    top = scores.amax(-1, keepdim=True)
    p = torch.exp(scores.double() - top.double()).float()
    total = p.double().sum(-1, keepdim=True)
    out = (p.half().double() @ vv) / total
    return out.float().half().transpose(1, 2).reshape(B, T, heads * dv)


def combine(attended: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, residual: torch.Tensor) -> torch.Tensor:
    """`linear(attended, combine_heads, bias, residual=x)` (model/fused_blocks.py:308-313): weight [K, N] fp16,
    accumulated in fp32 (fp64 here, then rounded), then + bias + residual, rounded to fp16."""
    acc = (attended.double() @ weight.double()).float()
    return ((acc + bias.float()) + residual.float()).half()


def embedding(boards: torch.Tensor, embed: torch.Tensor, position: torch.Tensor, table: torch.Tensor) -> torch.Tensor:
    """`input_embedding` (model/fused_blocks.py:370-406): embed[code] + position[t] + fp16(sum of the 23 feature rows in
    fp32), summed in fp32 and rounded to fp16 once. boards [B, 70] -> [B, 70, d] fp16."""
    boards = boards.long()
    B = boards.shape[0]
    rows = square_feature_indices(boards) + torch.from_numpy(ROW_OFFSETS)
    features = torch.zeros(B, NUM_SQUARES, table.shape[1], dtype=torch.float32)
    for f in range(rows.shape[-1]):
        features = features + table.float()[rows[..., f]]
    features = F.pad(features.half().float(), (0, 0, 0, TOKENS_PER_BOARD - NUM_SQUARES))
    total = embed.float()[boards] + position.float()[None]
    return (total + features).half()


def prepare(state: dict, settings: dict, weights: dict) -> dict:
    """What `int8_model` holds for a checkpoint (engine/inference.py:242-249,267-272; model/int8_blocks.py:254-272;
    model/fused_blocks.py:815-824): the stream scaled by 1/16, everything but the heads in fp16, down's scale times
    1/16, and the heads folded in fp64 then rounded. Every layer must have int8 weights."""
    g = geometry(settings)
    s = FP16_RESIDUAL_SCALE
    out = {"settings": settings, "g": g,
           "embed": (state["embed.weight"] * s).half(), "position": (state["position_embed"] * s).half(),
           "table": (state["square_features.table"] * s).half(), "templates": state["templates"].half(),
           "ln": state["ln.weight"].half(), "blocks": []}
    for i in range(g["layers"]):
        p = f"encoder.{i}."
        w = weights[i]
        out["blocks"].append({
            "dq": g["dqs"][i],
            "ln1": state[p + "ln1.weight"].half(), "ln2": state[p + "ln2.weight"].half(),
            "residual_scale": state[p + "residual_scale"].half(), "input_scale": state[p + "input_scale"].half(),
            "q_gain": state[p + "q_norm.weight"].half(), "k_gain": state[p + "k_norm.weight"].half(),
            "projection_bias": torch.cat([state[p + n + ".bias"] for n in ("Q", "K", "V", "template_mix")]).half(),
            "combine_heads": (state[p + "combine_heads.weight"] * s).half().t().contiguous(),
            "combine_heads_bias": (state[p + "combine_heads.bias"] * s).half(),
            "projection": w["projection"][0], "projection_scale": w["projection"][1].float(),
            "gate_up": w["gate_up"][0], "gate_up_scale": w["gate_up"][1].float(),
            "down": w["down"][0], "down_scale": (w["down"][1] * s).float()})
    from_w, from_b = state["from_projection.weight"].double(), state["from_projection.bias"].double()
    to_w, to_b = state["to_projection.weight"].double(), state["to_projection.bias"].double()
    scale = 1 / math.sqrt(g["d"])
    out["a_weight"] = (from_w.T @ to_w * scale).half()
    out["a_bias"] = (to_w.T @ from_b * scale).float()
    out["narrow_weight"] = torch.cat([(to_b @ from_w)[None] * scale, state["promotion_projection.weight"].double(),
                                      state["board_down_project.0.weight"].double()]).float()
    out["narrow_bias"] = torch.cat([(from_b @ to_b)[None] * scale, state["promotion_projection.bias"].double(),
                                    state["board_down_project.0.bias"].double()]).float()
    for name in ("eval_head.0.weight", "eval_head.0.bias", "eval_head.2.weight", "eval_head.2.bias"):
        out[name] = state[name].float()
    return out


def final_norm(x: torch.Tensor, gain: torch.Tensor, eps: float = EPS) -> torch.Tensor:
    """The final nn.RMSNorm in fp16 (model/fused_blocks.py:863): computed in fp32, rounded to fp16."""
    xf = x.float()
    inverse = torch.rsqrt((xf.double() * xf.double()).mean(-1, keepdim=True) + eps).float()
    return (xf * inverse * gain.float()).half()


def heads(x: torch.Tensor, prepared: dict) -> torch.Tensor:
    """The heads as the reference runs them on B200 (model/fused_blocks.py:863-874) and `answer_rows`
    (engine/inference.py:19-23): rows [B, 1969] fp32, the move logits then the expected score. fp32 products are
    exact-rounded here; the reference's tf32 matmuls only pass this within tolerance."""
    B = x.shape[0]
    y = final_norm(x, prepared["ln"])
    a = (y.double() @ prepared["a_weight"].double()).float() + prepared["a_bias"]
    yf = y.float()
    narrow = (yf.double() @ prepared["narrow_weight"].double().T + prepared["narrow_bias"].double()).float()
    squares = narrow[:, :NUM_SQUARES]
    logits = (a[:, :NUM_SQUARES].double() @ yf[:, :NUM_SQUARES].double().transpose(1, 2)).float() + squares[..., :1]
    combined = logits[:, torch.from_numpy(MOVE_FROM_SQUARES), torch.from_numpy(MOVE_TO_SQUARES)]
    promotions = squares[..., 1:5][:, torch.from_numpy(PROMOTION_TO_SQUARES), torch.from_numpy(PROMOTION_PIECES)]
    combined[:, torch.from_numpy(PROMOTION_MOVE_IDS)] += promotions
    compressed = F.gelu(narrow[..., 5:].double()).reshape(B, -1)
    hidden = F.gelu(compressed @ prepared["eval_head.0.weight"].double().T + prepared["eval_head.0.bias"].double())
    value = hidden @ prepared["eval_head.2.weight"].double().T + prepared["eval_head.2.bias"].double()
    score = torch.softmax(value, dim=-1) @ value_bin_centres(value.shape[-1]).double()
    return torch.cat([combined.float(), score.float()[:, None]], dim=1)


def block(prepared_block: dict, g: dict, x: torch.Tensor, templates: torch.Tensor, original: torch.Tensor,
          input_mixed: bool, next_scales: tuple | None) -> torch.Tensor:
    """`Int8Block.forward` (model/int8_blocks.py:274-288) on x [B, 70, d] fp16."""
    b = prepared_block
    B, T, d = x.shape
    M = B * T
    flat, orig = x.reshape(M, d), original.reshape(M, d)
    if not input_mixed:
        flat = mix(flat, orig, b["residual_scale"], b["input_scale"])
    q, s = norm_quant(flat, b["ln1"])
    projected = int8_linear(q, s, b["projection"], b["projection_scale"], bias=b["projection_bias"])
    attended = template_attention(projected.reshape(B, T, -1), templates, b["q_gain"], b["k_gain"], g["heads"], g["kv_heads"],
                                  b["dq"], g["dv"], g["templates"]).reshape(M, -1)
    flat = combine(attended, b["combine_heads"], b["combine_heads_bias"], flat)
    q, s = norm_quant(flat, b["ln2"])
    hidden = int8_linear(q, s, b["gate_up"], b["gate_up_scale"], gated=True)
    rotated, s = rotate_quant(hidden, b["down"].shape[1])
    if next_scales is None:
        out = int8_linear(rotated, s, b["down"], b["down_scale"], residual=flat)
    else:
        out = int8_linear(rotated, s, b["down"], b["down_scale"], residual=flat, original=orig,
                          residual_scale=next_scales[0], input_scale=next_scales[1])
    return out.reshape(B, T, d)


def int8_forward(prepared: dict, boards: torch.Tensor, return_stream: bool = False):
    """`FusedTransformer.forward` with every block an `Int8Block` (model/fused_blocks.py:856-874,
    model/int8_blocks.py:292-298): each down mixes the next block's input (`link_input_mixes`). Returns the answer rows
    [B, 1969] fp32 (and the last block's fp16 stream when asked)."""
    g = prepared["g"]
    x = embedding(boards, prepared["embed"], prepared["position"], prepared["table"])
    original = x
    blocks = prepared["blocks"]
    for i, b in enumerate(blocks):
        following = blocks[i + 1] if i + 1 < len(blocks) else None
        next_scales = (following["residual_scale"], following["input_scale"]) if following is not None else None
        x = block(b, g, x, prepared["templates"], original, input_mixed=i > 0, next_scales=next_scales)
    rows = heads(x, prepared)
    return (rows, x) if return_stream else rows
