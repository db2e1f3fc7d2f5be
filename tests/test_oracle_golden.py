"""The CPU oracle against the reference's own outputs (tests/golden/reference_golden.npz, written by
tests/golden/make_golden.py from the reference's model code and its Triton kernels run under the Triton interpreter).

The interpreter evaluates the reference's kernels in numpy, which never fuses a multiply-add; the GPU kernels and this
oracle do (model/int8_cuda.py:163-176). So epilogue outputs may differ from the fixtures by one fp16 step on a few
elements, and attention by the fp16 rounding of reordered fp32 sums. Integer work is bit-exact.
"""
import numpy as np
import pytest
import torch

from oracle import encoding, int8 as oi, model as om
from tests.conftest import SMALL, TINY


def t(array):
    return torch.from_numpy(np.ascontiguousarray(array))


def fp16_steps(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """How many fp16 steps apart two fp16 tensors are (exact on the integer view of same-sign values)."""
    ai, bi = a.view(torch.int16).int(), b.view(torch.int16).int()
    same_sign = (ai >= 0) == (bi >= 0)
    return torch.where(same_sign, (ai - bi).abs(), (a.float() - b.float()).abs().gt(0).int() * 1000)


def test_move_table_is_the_references(golden):
    assert encoding.NUM_MOVE_IDS == 1968 == len(golden["moves_from"])
    assert np.array_equal(encoding.MOVE_FROM_SQUARES, golden["moves_from"])
    assert np.array_equal(encoding.MOVE_TO_SQUARES, golden["moves_to"])
    assert np.array_equal(encoding.PROMOTION_MOVE_IDS, golden["promotion_ids"])
    assert np.array_equal(encoding.PROMOTION_TO_SQUARES, golden["promotion_to"])
    assert np.array_equal(encoding.PROMOTION_PIECES, golden["promotion_pieces"])


def test_square_features_are_the_references(golden):
    found = om.square_feature_indices(t(golden["feature_boards"]))
    assert np.array_equal(found.numpy(), golden["feature_indices"])
    assert np.array_equal(om.ROW_OFFSETS, golden["feature_row_offsets"])


@pytest.mark.parametrize("name, settings, seed", [("small", SMALL, 10), ("tiny", TINY, 11)])
def test_fp32_model_is_the_references(golden, name, settings, seed):
    with torch.no_grad():
        logits, values = om.fp32_forward(om.seeded_state_dict(settings, seed), settings, t(golden["fp32_boards"]))
    assert torch.allclose(logits, t(golden[f"fp32_{name}_logits"]), atol=2e-6, rtol=1e-5)
    assert torch.allclose(values, t(golden[f"fp32_{name}_values"]), atol=2e-6, rtol=1e-5)


def test_int8_weight_layout_is_the_references(golden):
    weights = oi.int8_weights(om.seeded_state_dict(SMALL, 10), SMALL, [0, 1])
    for layer in (0, 1):
        for name in ("projection", "gate_up", "down"):
            integers, scale = weights[layer][name]
            assert np.array_equal(integers.numpy(), golden[f"weights_{layer}_{name}_int8"]), (layer, name)
            assert np.allclose(scale.numpy(), golden[f"weights_{layer}_{name}_scale"], rtol=1e-7, atol=0), (layer, name)


@pytest.mark.parametrize("key", ["projection", "gate_up", "down", "mixing_down"])
def test_int8_linear_is_the_references(golden, key):
    g = lambda suffix: t(golden[f"linear_{key}_{suffix}"])
    kwargs = {}
    if key == "projection":
        kwargs["bias"] = g("bias")
    if key == "gate_up":
        kwargs["gated"] = True
    if key.endswith("down"):
        kwargs["residual"] = g("residual")
    if key == "mixing_down":
        scales = g("scales")
        kwargs.update(original=g("original"), residual_scale=scales[:1], input_scale=scales[1:])
    found = oi.int8_linear(g("x"), g("x_scale"), g("w"), g("w_scale"), **kwargs)
    expected = g("out")
    steps = fp16_steps(found, expected)
    assert steps.max() <= 1 and (steps > 0).float().mean() < 1e-3


def test_norm_quant_and_mix_are_the_references(golden):
    x, original, gain = t(golden["norm_x"]), t(golden["norm_original"]), t(golden["norm_gain"])
    q, scale = oi.norm_quant(x, gain)
    assert torch.equal(q, t(golden["norm_q"])) and torch.allclose(scale, t(golden["norm_scale"]), rtol=1e-6, atol=0)
    mixed = oi.mix(x, original, torch.tensor([0.8]).half(), torch.tensor([0.5]).half())
    assert torch.equal(mixed, t(golden["mix_out"]))
    q, scale = oi.norm_quant(mixed, gain)
    assert torch.equal(q, t(golden["mix_q"])) and torch.allclose(scale, t(golden["mix_scale"]), rtol=1e-6, atol=0)


@pytest.mark.parametrize("hidden, width", [(992, 1024), (320, 384)])
def test_rotate_quant_is_the_references(golden, hidden, width):
    q, scale = oi.rotate_quant(t(golden[f"rotate_{hidden}_h"]), width)
    assert torch.equal(q, t(golden[f"rotate_{hidden}_q"]))
    assert torch.allclose(scale, t(golden[f"rotate_{hidden}_scale"]), rtol=1e-6, atol=0)


@pytest.mark.parametrize("heads, kv_heads, dq", [(24, 12, 8), (24, 12, 16), (24, 12, 24), (4, 2, 16)])
def test_template_attention_is_the_references(golden, heads, kv_heads, dq):
    key = f"attention_{heads}_{kv_heads}_{dq}"
    g = lambda suffix: t(golden[f"{key}_{suffix}"])
    found = oi.template_attention(g("projected"), g("templates"), g("q_gain"), g("k_gain"), heads, kv_heads, dq, 32, 8)
    expected = g("out")
    assert (found.float() - expected.float()).abs().max() <= 1e-3
    assert (found == expected).float().mean() > 0.99


def test_combine_heads_linear_is_the_references_within_fp16_accumulation(golden):
    found = oi.combine(t(golden["combine_x"]), t(golden["combine_w"]), t(golden["combine_b"]), t(golden["combine_residual"]))
    # the reference accumulates this matmul in fp16; the oracle in fp32
    assert (found.float() - t(golden["combine_out"]).float()).abs().max() <= 8e-3


@pytest.mark.parametrize("name, settings, seed", [("small", SMALL, 10), ("tiny", TINY, 11)])
def test_int8_network_is_the_references(golden, name, settings, seed):
    state = om.seeded_state_dict(settings, seed)
    prepared = oi.prepare(state, settings, oi.int8_weights(state, settings))
    boards = t(golden["fp32_boards"][:4])
    embedding = oi.embedding(boards, prepared["embed"], prepared["position"], prepared["table"])
    assert torch.equal(embedding, t(golden[f"int8_{name}_embedding"]))
    rows = oi.int8_forward(prepared, boards)
    logits, values = t(golden[f"int8_{name}_logits"]), t(golden[f"int8_{name}_values"])
    assert (rows[:, :-1] - logits).abs().max() <= 1e-2
    assert (rows[:, -1] - om.expected_score(values)).abs().max() <= 1e-3
    assert torch.equal(rows[:, :-1].argmax(-1), logits.argmax(-1))
