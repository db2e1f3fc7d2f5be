"""Writes the golden fixtures under tests/golden/ from the reference's own code.

Run in the build container, where the reference is checked out (the path in
FRY_REFERENCE, or the default REFERENCE below):

    python tests/golden/make_golden.py

It imports the reference's `model/model.py`, `model/fused_blocks.py`,
`model/int8_blocks.py` and `engine/quantization.py`, with these stand-ins:

- python-chess is absent, so `tests/golden/chess_stub/chess` rebuilds the
  empty-board attack sets the move table is made from;
- there is no GPU, so the reference's Triton kernels run under the Triton
  interpreter (TRITON_INTERPRET=1), with the compute-capability queries
  answered as sm_120 (its tile tables are complete there), programmatic
  dependent launch off, and libdevice.rint given numpy's rint (round half to
  even, as rint is);
- `engine.quantization` imports its runtime neighbours only for names the
  functions used here never call, so those modules are replaced by empty ones.

The fixtures are inputs and outputs only. The synthetic weights are not
stored: `oracle.model.seeded_state_dict(settings, seed)` regenerates them and
the reference loads them with `load_state_dict`.
"""
import os
import sys
import types
from pathlib import Path
from types import SimpleNamespace

os.environ["TRITON_INTERPRET"] = "1"

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
REFERENCE = Path(os.environ.get("FRY_REFERENCE", "/root/reference"))
sys.path[:0] = [str(HERE / "chess_stub"), str(REFERENCE), str(REPO)]

import numpy as np
import torch

torch.cuda.get_device_capability = lambda device=None: (12, 0)
torch.cuda.get_device_properties = lambda device=None: SimpleNamespace(multi_processor_count=70, L2_cache_size=64 << 20)
torch.cuda.is_current_stream_capturing = lambda: False

import triton.language as tl
from triton.runtime.interpreter import TensorHandle

import model.encoding as ref_encoding
import model.fused_blocks as ref_fused
import model.int8_blocks as ref_int8
import model.model as ref_model

_no_pdl = lambda device: {"PDL": False, "launch_pdl": False}
ref_fused.dependent_launch = _no_pdl
ref_int8.dependent_launch = _no_pdl


def _rint(x):
    h = x.handle
    return tl.core.tensor(TensorHandle(np.rint(h.data).astype(h.data.dtype), h.dtype), x.type)


ref_int8.libdevice = SimpleNamespace(rint=_rint)
# quantize_blocks compiles the NVRTC small-batch kernels for the model's device; there is none here
ref_int8.kernels = lambda device: None

# engine.quantization's runtime neighbours, replaced by empty modules (gptq and compute_int8_weights use none of them)
_pgn = types.ModuleType("chess.pgn")
sys.modules["chess.pgn"] = _pgn
import chess as _chess
_chess.pgn = _pgn
_inference = types.ModuleType("engine.inference")
_inference.FP16_RESIDUAL_SCALE = 1 / 16
_inference.answer_rows = None
_inference.fp16_model = None
sys.modules["engine.inference"] = _inference
import engine.quantization as ref_quantization

from oracle.model import seeded_state_dict
from seeded_boards import golden_boards  # noqa: E402  (tests/golden, on the path above)

SMALL = {"d_model": 128, "num_layers": 3, "n_heads": 4, "kv_heads": 2, "qk_ratio": [0.25, 0.5, 0.75], "mlp_hidden": 320, "value_bins": 16}
# config 0's network in Fry's geometry: d 256, 8 query heads of 32, 4 key/value heads, dq 8/16/24, SwiGLU 1024, 128 bins
TINY = {"d_model": 256, "num_layers": 6, "n_heads": 8, "kv_heads": 4, "qk_ratio": [0.25, 0.5, 0.75] * 2, "mlp_hidden": 1024,
        "value_bins": 128}


def reference_model(settings: dict, seed: int) -> ref_model.ChessTransformer:
    model = ref_model.ChessTransformer(**settings).eval()
    model.load_state_dict(seeded_state_dict(settings, seed))
    return model


def fp16_int8_model(settings: dict, seed: int, weights: dict) -> torch.nn.Module:
    """`engine.inference.int8_model` (engine/inference.py:242-249,267-272) without the checkpoint file."""
    model = reference_model(settings, seed).scale_residual_stream(1 / 16).half_except_heads(torch.float16)
    return ref_int8.quantize_blocks(ref_fused.FusedTransformer(model), weights, 1 / 16)


def rtn_weights(model: ref_model.ChessTransformer, layers: list[int]) -> dict:
    """The reference's own weight layout (engine/quantization.py:124-140) with gptq given an identity Hessian, which
    rounds to nearest (tests/test_int8.py:35-41)."""
    real = ref_quantization.gptq
    ref_quantization.gptq = lambda weight, hessian: real(weight, torch.eye(weight.shape[1], dtype=torch.float64))
    try:
        # fp64 but the heads, as int8_weights loads the model (engine/quantization.py:200-201)
        everything = ref_quantization.compute_int8_weights(model.half_except_heads(torch.float64), torch.from_numpy(golden_boards(8, 99)).long())
    finally:
        ref_quantization.gptq = real
    return {layer: everything[layer] for layer in layers if layer in everything}


def main() -> None:
    torch.manual_seed(0)
    out = {}

    # encoding constants (model/encoding.py:25-69)
    out["moves_from"] = np.array(ref_encoding.MOVE_FROM_SQUARES)
    out["moves_to"] = np.array(ref_encoding.MOVE_TO_SQUARES)
    out["promotion_ids"] = np.array(ref_encoding.PROMOTION_MOVE_IDS)
    out["promotion_to"] = np.array(ref_encoding.PROMOTION_TO_SQUARES)
    out["promotion_pieces"] = np.array(ref_encoding.PROMOTION_PIECES)

    # square features (model/model.py:147-169) on random boards and a few crafted ones
    boards = golden_boards(96, 1)
    features = ref_model.SquareFeatures(8)
    out["feature_boards"] = boards
    out["feature_indices"] = features.indices(torch.from_numpy(boards).long()).numpy().astype(np.int16)
    out["feature_row_offsets"] = features.row_offsets.numpy()

    # the fp32 model (model/model.py:245-270)
    boards16 = golden_boards(16, 2)
    out["fp32_boards"] = boards16
    for name, settings, seed in (("small", SMALL, 10), ("tiny", TINY, 11)):
        with torch.no_grad():
            logits, values = reference_model(settings, seed)(torch.from_numpy(boards16).long())
        out[f"fp32_{name}_logits"] = logits.numpy()
        out[f"fp32_{name}_values"] = values.numpy()

    # int8 weight layout (engine/quantization.py:124-140) for SMALL seed 10, all layers but the last
    weights = rtn_weights(reference_model(SMALL, 10), [0, 1])
    for layer, matmuls in weights.items():
        for name, (integers, scale) in matmuls.items():
            out[f"weights_{layer}_{name}_int8"] = integers.numpy()
            out[f"weights_{layer}_{name}_scale"] = scale.numpy()

    # kernel-level goldens from the reference's Triton kernels under the interpreter
    g = torch.Generator().manual_seed(3)
    rows, width = 2 * 70, 200
    for matmul in ("projection", "gate_up", "down", "mixing down"):
        down, gated = matmul.endswith("down"), matmul == "gate_up"
        depth = 1024 if down else 256
        x = torch.randint(-127, 128, (rows, depth), generator=g, dtype=torch.int8)
        x_scale = torch.rand(rows, generator=g) / 100
        weight = torch.randint(-127, 128, (2 * width if gated else width, depth), generator=g, dtype=torch.int8)
        weight_scale = torch.rand(len(weight), generator=g) / 100
        bias = torch.randn(width, generator=g).half() if matmul == "projection" else None
        residual = torch.randn(rows, width, generator=g).half() if down else None
        mix = (torch.randn(rows, width, generator=g).half(), torch.tensor([0.9]).half(), torch.tensor([0.3]).half()) \
            if matmul == "mixing down" else (None, None, None)
        result = ref_int8.launch_int8_linear(x, x_scale, weight, weight_scale, bias, residual, gated, *mix, (32, 64, 64, 4, 4))
        key = matmul.replace(" ", "_")
        out[f"linear_{key}_x"], out[f"linear_{key}_x_scale"] = x.numpy(), x_scale.numpy()
        out[f"linear_{key}_w"], out[f"linear_{key}_w_scale"] = weight.numpy(), weight_scale.numpy()
        if bias is not None:
            out[f"linear_{key}_bias"] = bias.numpy()
        if residual is not None:
            out[f"linear_{key}_residual"] = residual.numpy()
        if mix[0] is not None:
            out[f"linear_{key}_original"] = mix[0].numpy()
            out[f"linear_{key}_scales"] = torch.cat([mix[1], mix[2]]).numpy()
        out[f"linear_{key}_out"] = result.numpy()

    x = (torch.randn(2, 70, 192, generator=g) * 4).half()
    original = torch.randn(2, 70, 192, generator=g).half()
    gain = (torch.rand(192, generator=g) + 0.5).half()
    scales = torch.tensor([0.8, 0.5]).half()
    q, s = ref_int8.norm_quant(x, gain, 1e-5)
    mixed, mq, ms = ref_int8.mix_norm_quant(x, original, scales[:1], scales[1:], gain, 1e-5)
    out.update(norm_x=x.numpy(), norm_original=original.numpy(), norm_gain=gain.numpy(), norm_q=q.numpy(), norm_scale=s.numpy(),
               mix_out=mixed.numpy(), mix_q=mq.numpy(), mix_scale=ms.numpy())

    for hidden, width in ((992, 1024), (320, 384)):
        h = torch.randn(1, 70, hidden, generator=g).half()
        rq, rs = ref_int8.rotate_quant(h, ref_int8.hadamard(32).half(), width)
        out[f"rotate_{hidden}_h"], out[f"rotate_{hidden}_q"], out[f"rotate_{hidden}_scale"] = h.numpy(), rq.numpy(), rs.numpy()

    for heads, kv_heads, dq, positions in ((24, 12, 8, 1), (24, 12, 16, 1), (24, 12, 24, 1), (4, 2, 16, 3)):
        projected = torch.randn(positions, 70, heads * dq + kv_heads * dq + kv_heads * 32 + heads * 8, generator=g).half()
        templates = (torch.randn(8, 64, 64, generator=g) / 2).half()
        q_gain, k_gain = (1 + torch.randn(2, dq, generator=g) / 10).half()
        attended = ref_fused.template_attention(projected, templates, q_gain, k_gain, heads, kv_heads, dq, 32, 8, 1e-5)
        key = f"attention_{heads}_{kv_heads}_{dq}"
        out.update({f"{key}_projected": projected.numpy(), f"{key}_templates": templates.numpy(), f"{key}_q_gain": q_gain.numpy(),
                    f"{key}_k_gain": k_gain.numpy(), f"{key}_out": attended.numpy()})

    attended = torch.randn(rows, 128, generator=g).half()
    combine_w = (torch.randn(128, 128, generator=g) / 16).half()
    combine_b = (torch.randn(128, generator=g) / 16).half()
    residual = torch.randn(rows, 128, generator=g).half()
    out.update(combine_x=attended.numpy(), combine_w=combine_w.numpy(), combine_b=combine_b.numpy(), combine_residual=residual.numpy(),
               combine_out=ref_fused.linear(attended, combine_w, combine_b, residual=residual).numpy())

    # end to end: the reference's int8 model on SMALL and TINY with every block int8 (round-to-nearest weights),
    # and on SMALL in the reference's own layout (the last block fp16)
    for name, settings, seed in (("small", SMALL, 10), ("tiny", TINY, 11)):
        layers = list(range(settings["num_layers"]))
        weights = rtn_weights(reference_model(settings, seed), layers)
        weights[layers[-1]] = rtn_last_layer(reference_model(settings, seed), layers[-1])
        with torch.no_grad():
            network = fp16_int8_model(settings, seed, weights)
            embedding = network.input_embedding(torch.from_numpy(boards16[:4]).long())
            logits, values = network(torch.from_numpy(boards16[:4]).long())
        out[f"int8_{name}_embedding"] = embedding.numpy()
        out[f"int8_{name}_logits"] = logits.numpy()
        out[f"int8_{name}_values"] = values.numpy()
    with torch.no_grad():
        network = fp16_int8_model(SMALL, 10, rtn_weights(reference_model(SMALL, 10), [0, 1]))
        logits, values = network(torch.from_numpy(boards16[:4]).long())
    out["int8_small_layout_logits"], out["int8_small_layout_values"] = logits.numpy(), values.numpy()

    np.savez_compressed(HERE / "reference_golden.npz", **out)
    print(f"wrote {HERE / 'reference_golden.npz'}: {len(out)} arrays")


def rtn_last_layer(model: ref_model.ChessTransformer, layer: int) -> dict:
    """The last block's weights in the same layout: compute_int8_weights leaves it out (FP16_LAST_LAYERS), so it is
    rounded here with FP16_LAST_LAYERS set to 0."""
    kept = ref_quantization.FP16_LAST_LAYERS
    ref_quantization.FP16_LAST_LAYERS = 0
    try:
        return rtn_weights(model, [layer])[layer]
    finally:
        ref_quantization.FP16_LAST_LAYERS = kept


if __name__ == "__main__":
    main()
