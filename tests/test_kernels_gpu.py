"""Each kernel of libfry_b200.so through the C ABI (chess_transformer_b200.ops) against the CPU oracle and against the
reference's own outputs (tests/golden/reference_golden.npz). Tolerances are the reference's own where it states them
(tests/test_int8.py:59-90,246-281; tests/test_attention_cuda.py:63-79; tests/test_inference.py:325-384).
int32 sums are compared bit for bit."""
import numpy as np
import pytest
import torch

from chess_transformer_b200 import ops
from chess_transformer_b200.build import build
from oracle import int8 as oi, model as om

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def built():
    build()


def t(array, device="cuda"):
    return torch.from_numpy(np.ascontiguousarray(array)).to(device)


def fp16_steps(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """|a - b| in units of the fp16 spacing at the larger of |a|, |b| (subnormal spacing 2^-24 near zero)."""
    a, b = a.cpu().double(), b.cpu().double()
    larger = torch.maximum(a.abs(), b.abs()).clamp(min=2.0 ** -14)
    spacing = torch.exp2(torch.floor(torch.log2(larger)) - 10)
    return ((a - b).abs() / spacing).round().int()


def int8_operands(M, N, K, seed, gated=False):
    g = torch.Generator().manual_seed(seed)
    x = torch.randint(-127, 128, (M, K), generator=g, dtype=torch.int8)
    w = torch.randint(-127, 128, (2 * N if gated else N, K), generator=g, dtype=torch.int8)
    xs = torch.rand(M, generator=g) / 100
    ws = torch.rand(len(w), generator=g) / 100
    return x, w, xs, ws, g


# shapes: partial tiles in M and N, the Fry projection/gate_up/down/attention-out widths, small and large M
@pytest.mark.parametrize("M, N, K", [(70, 200, 256), (210, 200, 1024), (4480, 864, 768), (4480, 1152, 768), (4480, 1440, 768),
                                     (1400, 992, 768), (4480, 768, 1024), (17920, 768, 1024), (1, 8, 16)])
def test_int8_sums_are_bit_exact(M, N, K):
    x, w, _, _, _ = int8_operands(M, N, K, seed=M + N + K)
    found = ops.int8_matmul_i32(x.cuda(), w.cuda()).cpu()
    assert torch.equal(found, oi.int8_matmul(x, w))


@pytest.mark.parametrize("key", ["projection", "gate_up", "down", "mixing_down"])
def test_int8_linear_is_the_references(golden, key):
    g = lambda suffix: t(golden[f"linear_{key}_{suffix}"])
    kwargs = {}
    if key == "projection":
        kwargs["bias"] = g("bias")
    if key.endswith("down"):
        kwargs["residual"] = g("residual")
    if key == "mixing_down":
        scales = g("scales")
        kwargs.update(original=g("original"), residual_scale=scales[:1].contiguous(), input_scale=scales[1:].contiguous())
    found = ops.int8_linear(g("x"), g("x_scale"), g("w"), g("w_scale"), kwargs.pop("bias", None), kwargs.pop("residual", None),
                            key == "gate_up", key, **kwargs)
    expected = g("out")
    steps = fp16_steps(found, expected)
    # the reference's kernels fuse the epilogue's multiply-adds as these do; the interpreter that wrote the fixtures
    # does not, so a few elements differ by one fp16 step
    assert steps.max() <= 1 and (steps > 0).float().mean() < 2e-3
    # and the reference's own criterion: the dequantised fp64 matmul plus epilogue (tests/test_int8.py:59-90)
    x, xs, w, ws = (golden[f"linear_{key}_{s}"] for s in ("x", "x_scale", "w", "w_scale"))
    projected = (x.astype(np.float64) * xs[:, None].astype(np.float64)) @ (w.astype(np.float64) * ws[:, None].astype(np.float64)).T
    if key == "projection":
        exact = projected + golden["linear_projection_bias"].astype(np.float64)
    elif key == "gate_up":
        gate, up = np.split(projected, 2, axis=1)
        exact = gate / (1 + np.exp(-gate)) * up
    else:
        exact = projected + golden[f"linear_{key}_residual"].astype(np.float64)
    if key == "mixing_down":
        rs, is_ = golden["linear_mixing_down_scales"].astype(np.float64)
        exact = rs * exact.astype(np.float16).astype(np.float64) + is_ * golden["linear_mixing_down_original"].astype(np.float64)
    assert np.allclose(found.cpu().double().numpy(), exact, atol=1e-3, rtol=2e-3)


# 17920 and 19001 rows: 140 and 149 row blocks over the SMs, so some CTAs take two (the last block partial)
@pytest.mark.parametrize("M", [5, 70, 4480, 17920, 19001])
@pytest.mark.parametrize("epilogue, N, K", [("bias", 864, 768), ("bias", 1152, 768), ("bias", 1440, 768), ("gated", 992, 768),
                                            ("residual", 768, 1024), ("mixing", 768, 1024)])
def test_int8_linear_is_the_oracle_on_fry_shapes(M, epilogue, N, K):
    x, w, xs, ws, g = int8_operands(M, N, K, seed=M * 7 + N, gated=epilogue == "gated")
    bias = torch.randn(N, generator=g).half() if epilogue == "bias" else None
    residual = torch.randn(M, N, generator=g).half() if epilogue in ("residual", "mixing") else None
    mix = (torch.randn(M, N, generator=g).half(), torch.tensor([0.8]).half(), torch.tensor([0.5]).half()) if epilogue == "mixing" else None
    cuda = lambda v: v.cuda() if v is not None else None
    found = ops.int8_linear(x.cuda(), xs.cuda(), w.cuda(), ws.cuda(), cuda(bias), cuda(residual), epilogue == "gated", epilogue,
                            *(tuple(cuda(v) for v in mix) if mix else ())).cpu()
    expected = oi.int8_linear(x, xs, w, ws, bias=bias, residual=residual, gated=epilogue == "gated",
                              **({"original": mix[0], "residual_scale": mix[1], "input_scale": mix[2]} if mix else {}))
    steps = fp16_steps(found, expected)
    # bias/residual/mixing follow the oracle's op order exactly; the gate's sigmoid uses the hardware 2^x
    assert steps.max() <= (1 if epilogue == "gated" else 0)


# the fused norm: units of a row block's column tiles (1, 5 and 70 rows: one row block split over up to 23 CTAs; 4480: 35
# blocks, 4 groups; 17920: 140 blocks, one CTA each; 19001: 149 blocks, a CTA takes two, the last one partial)
@pytest.mark.parametrize("M", [1, 5, 70, 4480, 17920, 19001])
@pytest.mark.parametrize("epilogue, N", [("bias", 864), ("bias", 1152), ("bias", 1440), ("gated", 992), ("gated", 1024)])
def test_int8_linear_normed_is_norm_quant_then_int8_linear(M, epilogue, N):
    g = torch.Generator().manual_seed(M + N)
    K = 768
    x = (torch.randn(M, K, generator=g) * 3).half().cuda()
    gain = (torch.rand(K, generator=g) + 0.5).half().cuda()
    gated = epilogue == "gated"
    w = torch.randint(-127, 128, (2 * N if gated else N, K), generator=g, dtype=torch.int8).cuda()
    ws = (torch.rand(len(w), generator=g) / 100).cuda()
    bias = None if gated else torch.randn(N, generator=g).half().cuda()
    found = ops.int8_linear_normed(x, gain, 1e-5, w, ws, bias, gated)
    # the same bits as the two kernels it replaces
    q, scale = ops.norm_quant(x, gain, 1e-5)
    pair = ops.int8_linear(q, scale, w, ws, bias, None, gated, epilogue)
    assert torch.equal(found.cpu(), pair.cpu())
    # and the oracle's: its int8_linear on those int8 rows (the gate's sigmoid one fp16 step apart at most), its norm_quant
    # within one int8 step (rsqrt)
    expected = oi.int8_linear(q.cpu(), scale.cpu(), w.cpu(), ws.cpu(), bias=None if bias is None else bias.cpu(), gated=gated)
    assert fp16_steps(found, expected).max() <= (1 if gated else 0)
    oq, _ = oi.norm_quant(x.cpu(), gain.cpu())
    assert (q.cpu().int() - oq.int()).abs().max() <= 1


def test_int8_linear_normed_refuses_other_widths():
    x = torch.zeros(70, 512, dtype=torch.float16, device="cuda")
    with pytest.raises(Exception, match="K = 768"):
        ops.int8_linear_normed(x, x[0], 1e-5, torch.zeros(64, 512, dtype=torch.int8, device="cuda"),
                               torch.ones(64, device="cuda"), None, False)


# the attention-out linear with ln2's norm in its epilogue: a cluster of N / 256 CTAs a row block (1 to 4); 17920 rows: 140
# row blocks, more than the clusters the device holds at once, so clusters take several
@pytest.mark.parametrize("M, N", [(1, 768), (70, 768), (4480, 768), (17920, 768), (19001, 768), (300, 256), (300, 1024)])
def test_linear_norm_quant_is_linear_then_norm_quant(M, N):
    g = torch.Generator().manual_seed(M + N)
    K = 768
    x = torch.randn(M, K, generator=g).half().cuda()
    weight = (torch.randn(K, N, generator=g) / 16).half().cuda()
    bias = (torch.randn(N, generator=g) / 16).half().cuda()
    residual = (torch.randn(M, N, generator=g) * 2).half().cuda()
    gain = (torch.rand(N, generator=g) + 0.5).half().cuda()
    out, q, scale = ops.linear_norm_quant(x, weight, bias, residual, gain, 1e-5)
    expected = ops.linear(x, weight, bias, residual)
    assert torch.equal(out.cpu(), expected.cpu())  # the same epilogue, bit for bit
    eq, escale = ops.norm_quant(expected, gain, 1e-5)
    # the squares summed in another order and absmax from max|out * gain|: scales within fp32 rounding, an int8 value one
    # step apart now and then
    assert torch.allclose(scale.cpu(), escale.cpu(), rtol=2e-6, atol=0)
    difference = (q.cpu().int() - eq.cpu().int()).abs()
    assert difference.max() <= 1 and (difference > 0).float().mean() < 1e-3
    # and the reference's own criterion (tests/test_int8.py:246-264) against the fp32 RMSNorm of the fp16 output
    normed = torch.nn.functional.rms_norm(expected.float().cpu(), (N,), gain.float().cpu(), 1e-5)
    step = normed.abs().amax(-1) / 127
    assert ((q.cpu().float() * scale.cpu()[:, None] - normed).abs() <= 0.501 * step[:, None] + 1e-6).all()


# 17920 and 19001 rows take CTA pairs (at 19001 the last 256-row tile holds 57 real rows, all in its first CTA)
@pytest.mark.parametrize("M, N, K", [(70, 200, 128), (4480, 768, 768), (17920, 768, 768), (19001, 768, 768)])
def test_fp16_linear_is_the_oracle(M, N, K):
    g = torch.Generator().manual_seed(N)
    x = torch.randn(M, K, generator=g).half()
    weight = (torch.randn(K, N, generator=g) / 16).half()
    bias = (torch.randn(N, generator=g) / 16).half()
    residual = torch.randn(M, N, generator=g).half()
    found = ops.linear(x.cuda(), weight.cuda(), bias.cuda(), residual.cuda()).cpu()
    expected = oi.combine(x, weight, bias, residual)
    # fp32 sums in another order than the oracle's exact one: one fp16 step, plus the fp32 rounding of sums of
    # magnitude ~1 where acc + bias + residual cancels towards zero
    assert ((found.float() - expected.float()).abs() <= expected.float().abs() * 2 ** -10 + 2e-5).all()
    found32 = ops.linear(x.cuda(), weight.cuda(), bias.float().cuda(), accumulate_fp32=True).cpu()
    exact = (x.double() @ weight.double() + bias.double()).float()
    assert found32.dtype == torch.float32 and torch.allclose(found32, exact, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("M", [70, 4480, 17920])
def test_fp16_gated_and_mixing_linears_are_their_fp32_epilogues(M):
    # the fp16 blocks' forms (model/fused_blocks.py:209-225): the reference's epilogue in fp32 on exact (fp64) sums
    g = torch.Generator().manual_seed(M)
    K, hidden, D = 768, 992, 768
    x = torch.randn(M, K, generator=g).half()
    gate_up = (torch.randn(K, 2 * hidden, generator=g) / 16).half()
    bias = (torch.randn(hidden, generator=g) / 4).half()
    hidden_out = ops.linear(x.cuda(), gate_up.cuda(), bias.cuda(), gated=True).cpu()
    sums = x.double() @ gate_up.double()
    gate, up = (sums[:, :hidden] + bias.double()).float(), sums[:, hidden:].float()
    expected = (gate * torch.sigmoid(gate) * up).half()
    # fp32 sums in another order and the sigmoid from the 2^x instruction: within an fp16 step and a little absolute slack
    assert ((hidden_out.float() - expected.float()).abs() <= expected.float().abs() * 2 ** -10 + 1e-4).all()

    h = (torch.randn(M, hidden, generator=g) / 2).half()
    down = (torch.randn(hidden, D, generator=g) / 32).half()
    residual, original = torch.randn(M, D, generator=g).half(), torch.randn(M, D, generator=g).half()
    scales = torch.tensor([0.8, 0.5]).half()
    mixed = ops.linear(h.cuda(), down.cuda(), None, residual.cuda(), original=original.cuda(), residual_scale=scales[:1].cuda(),
                       input_scale=scales[1:].cuda()).cpu()
    stream = ((h.double() @ down.double()).float() + residual.float()).half().float()
    rs, is_ = scales.float()
    expected = (rs * stream + is_ * original.float()).half()
    assert ((mixed.float() - expected.float()).abs() <= expected.float().abs() * 2 ** -9 + 2e-3).all()


def test_combine_linear_is_the_references_within_its_fp16_accumulation(golden):
    found = ops.linear(t(golden["combine_x"]), t(golden["combine_w"]), t(golden["combine_b"]), t(golden["combine_residual"])).cpu()
    assert (found.float() - torch.from_numpy(golden["combine_out"]).float()).abs().max() <= 8e-3


def test_norm_quant_and_mix_are_the_references(golden):
    x, original, gain = t(golden["norm_x"]), t(golden["norm_original"]), t(golden["norm_gain"])
    q, scale = ops.norm_quant(x, gain, 1e-5)
    assert torch.equal(q.cpu(), torch.from_numpy(golden["norm_q"]))
    assert torch.allclose(scale.cpu(), torch.from_numpy(golden["norm_scale"]), rtol=1e-6, atol=0)
    scales = torch.tensor([0.8, 0.5]).half().cuda()
    mixed, mq, ms = ops.mix_norm_quant(x, original, scales[:1], scales[1:], gain, 1e-5)
    assert torch.equal(mixed.cpu(), torch.from_numpy(golden["mix_out"]))
    assert torch.equal(mq.cpu(), torch.from_numpy(golden["mix_q"]))


@pytest.mark.parametrize("D, rows", [(768, 4480), (128, 210), (256, 70)])
def test_norm_quant_rounds_the_rmsnorm(D, rows):
    # tests/test_int8.py:246-264: scales within rtol 1e-5 of absmax/127 and every element within 0.501 steps
    g = torch.Generator().manual_seed(D)
    x = (torch.randn(rows, D, generator=g) * 4).half()
    gain = (torch.rand(D, generator=g) + 0.5).half()
    q, scale = ops.norm_quant(x.cuda(), gain.cuda(), 1e-5)
    q, scale = q.cpu(), scale.cpu()
    normed = torch.nn.functional.rms_norm(x.float(), (D,), gain.float(), 1e-5)
    step = normed.abs().amax(-1) / 127
    assert torch.allclose(scale, step, rtol=1e-5)
    assert ((q.float() * scale[:, None] - normed).abs() <= 0.501 * step[:, None]).all()
    oq, _ = oi.norm_quant(x, gain)
    assert (q.int() - oq.int()).abs().max() <= 1 and (q != oq).float().mean() < 1e-3


@pytest.mark.parametrize("hidden, width", [(992, 1024), (320, 384)])
def test_rotate_quant_is_the_references(golden, hidden, width):
    q, scale = ops.rotate_quant(t(golden[f"rotate_{hidden}_h"]), oi.hadamard(32).half().cuda(), width)
    assert torch.equal(q.cpu(), torch.from_numpy(golden[f"rotate_{hidden}_q"]))
    assert torch.allclose(scale.cpu(), torch.from_numpy(golden[f"rotate_{hidden}_scale"]), rtol=1e-6, atol=0)


def test_rotate_quant_rounds_the_rotated_rows():
    # tests/test_int8.py:267-281 on a full batch: padded columns exactly 0, every element within 0.501 steps
    h = torch.randn(4480, 992, generator=torch.Generator().manual_seed(1)).half()
    q, scale = ops.rotate_quant(h.cuda(), oi.hadamard(32).half().cuda(), 1024)
    q, scale = q.cpu(), scale.cpu()
    rotation = torch.block_diag(*[oi.hadamard(32)] * 32)
    rotated = torch.nn.functional.pad(h.float(), (0, 32)) @ rotation
    step = rotated.abs().amax(-1) / 127
    assert torch.allclose(scale, step, rtol=1e-5)
    assert ((q.float() * scale[:, None] - rotated).abs() <= 0.501 * step[:, None]).all()


@pytest.mark.parametrize("heads, kv_heads, dq", [(24, 12, 8), (24, 12, 16), (24, 12, 24), (4, 2, 16)])
def test_template_attention_is_the_references(golden, heads, kv_heads, dq):
    key = f"attention_{heads}_{kv_heads}_{dq}"
    g = lambda suffix: t(golden[f"{key}_{suffix}"])
    found = ops.template_attention(g("projected"), g("templates"), g("q_gain"), g("k_gain"), heads, kv_heads, dq, 32, 8, 1e-5).cpu()
    expected = torch.from_numpy(golden[f"{key}_out"])
    assert (found.float() - expected.float()).abs().max() <= 4e-3


@pytest.mark.parametrize("dq", [8, 16, 24])
@pytest.mark.parametrize("positions", [1, 5, 37, 64])
def test_template_attention_is_the_attention_in_fp32(dq, positions):
    # tests/test_attention_cuda.py:51-71: against fp32 torch with atol 1e-2; and against the oracle's rounding points
    g = torch.Generator().manual_seed(positions * 31 + dq)
    projected = torch.randn(positions, 70, 36 * dq + 576, generator=g).half()
    templates = (torch.randn(8, 64, 64, generator=g) / 2).half()
    q_gain, k_gain = (1 + torch.randn(2, dq, generator=g) / 10).half()
    found = ops.template_attention(projected.cuda(), templates.cuda(), q_gain.cuda(), k_gain.cuda(), 24, 12, dq, 32, 8, 1e-5).cpu()
    expected = oi.template_attention(projected, templates, q_gain, k_gain, 24, 12, dq, 32, 8)
    # a template bias or probability whose fp32 sum sits on an fp16 rounding boundary may round the other way than the
    # oracle's exactly-rounded sum: the reference allows its CUDA and Triton kernels 4e-3 (tests/test_attention_cuda.py:74-79)
    difference = (found.float() - expected.float()).abs()
    assert difference.max() <= 4e-3 and (difference > 1e-3).float().mean() < 1e-3
    q, k, v, c = projected.float().split([24 * dq, 12 * dq, 12 * 32, 24 * 8], dim=-1)
    F = torch.nn.functional
    qn = F.rms_norm(q.reshape(positions, 70, 24, dq), (dq,), q_gain.float(), 1e-5).transpose(1, 2)
    kn = F.rms_norm(k.reshape(positions, 70, 12, dq), (dq,), k_gain.float(), 1e-5).transpose(1, 2).repeat_interleave(2, 1)
    vv = v.reshape(positions, 70, 12, 32).transpose(1, 2).repeat_interleave(2, 1)
    bias = torch.einsum("biht,tij->bhij", c[:, :64].reshape(positions, 64, 24, 8), templates.float())
    scores = qn @ kn.transpose(-2, -1) / dq ** 0.5 + F.pad(bias, (0, 6, 0, 6))
    fp32 = (torch.softmax(scores, -1) @ vv).transpose(1, 2).reshape(positions, 70, 768)
    assert torch.allclose(found.float(), fp32, atol=1e-2)


def test_template_attention_reads_the_templates_and_their_coefficients():
    # tests/test_attention_cuda.py:100-107
    g = torch.Generator().manual_seed(5)
    projected = torch.randn(8, 70, 36 * 16 + 576, generator=g).half().cuda()
    templates = (torch.randn(8, 64, 64, generator=g) / 2).half().cuda()
    gains = torch.ones(16).half().cuda()
    run = lambda p, tm: ops.template_attention(p, tm, gains, gains, 24, 12, 16, 32, 8, 1e-5)
    without_bias = run(projected, torch.zeros_like(templates))
    mixed = projected.clone()
    mixed[..., -24 * 8:] = 0
    assert torch.equal(without_bias, run(mixed, templates))
    assert (run(projected, templates).float() - without_bias.float()).abs().max() > 0.05


@pytest.mark.parametrize("name", ["small", "tiny"])
def test_board_embedding_is_the_references(golden, name):
    from tests.conftest import SMALL, TINY
    settings, seed = {"small": (SMALL, 10), "tiny": (TINY, 11)}[name]
    prepared = oi.prepare(om.seeded_state_dict(settings, seed), settings, oi.int8_weights(om.seeded_state_dict(settings, seed), settings))
    boards = t(golden["fp32_boards"][:4]).long()
    found = ops.board_embedding(boards, prepared["embed"].cuda(), prepared["position"].cuda(), prepared["table"].cuda()).cpu()
    assert torch.equal(found, torch.from_numpy(golden[f"int8_{name}_embedding"]))


def test_board_embedding_finds_the_square_features_exactly():
    # tests/test_inference.py:325-351: whole-number tables make every sum exact (and small enough that fp16 holds them)
    from chess_transformer_b200.boards import random_boards
    g = torch.Generator().manual_seed(0)
    d = 96
    embed, position = torch.randint(-32, 32, (81, d), generator=g).half(), torch.randint(-32, 32, (70, d), generator=g).half()
    table = torch.randint(-32, 32, (1735, d), generator=g).half()
    boards = torch.from_numpy(random_boards(600, 3)).long()
    found = ops.board_embedding(boards.cuda(), embed.cuda(), position.cuda(), table.cuda()).cpu()
    rows = om.square_feature_indices(boards) + torch.from_numpy(om.ROW_OFFSETS)
    features = torch.nn.functional.pad(table.double()[rows].sum(-2), (0, 0, 0, 6))
    expected = (embed.double()[boards] + position.double() + features).half()
    assert torch.equal(found, expected)


@pytest.mark.parametrize("boards", [1, 5, 71])
def test_heads_are_the_oracles(boards):
    from tests.conftest import SMALL
    settings = {**SMALL, "d_model": 128}
    state = om.seeded_state_dict(settings, 4, from_scale=8.0)
    prepared = oi.prepare(state, settings, oi.int8_weights(state, settings))
    stream = (torch.randn(boards, 70, 128, generator=torch.Generator().manual_seed(boards)) / 4).half()
    a_weight_nk = prepared["a_weight"].t().contiguous()
    found = ops.heads(stream.cuda(), prepared["ln"].cuda(), a_weight_nk.cuda(), prepared["a_bias"].cuda(), prepared["narrow_weight"].cuda(),
                      prepared["narrow_bias"].cuda(), prepared["eval_head.0.weight"].cuda(), prepared["eval_head.0.bias"].cuda(),
                      prepared["eval_head.2.weight"].cuda(), prepared["eval_head.2.bias"].cuda(), 1e-5).cpu()
    expected = oi.heads(stream, prepared)
    assert found.shape == (boards, 1969)
    # the final norm's output is rounded to fp16 (the reference's B200 path runs it as an fp16 module); an element whose
    # fp32 value sits on a rounding boundary may round one step apart from the oracle's, which moves its row's logits by
    # ~1e-4. Everything after it is fp32-grade (split-fp16 products, fp32 sums).
    difference = (found[:, :-1] - expected[:, :-1]).abs()
    assert difference.max() <= 2e-3 and difference.median() <= 1e-5
    assert torch.allclose(found[:, -1], expected[:, -1], rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("dq", [8, 16, 24])
@pytest.mark.parametrize("boards", [1, 5, 64, 256])
def test_the_q_k_norm_in_the_projection_epilogue_gives_the_attentions_own_bits(dq, boards):
    # the forward's fused pair (fry_int8_linear_qk_norm, then fry_template_attention_normed) against the
    # plain pair (fry_int8_linear, then fry_template_attention, which normalises queries and keys itself), at Fry's
    # geometry: the value and template-mix columns and the attention's output are the same bits
    import ctypes
    from chess_transformer_b200.library import library
    lib = library()
    heads, kv_heads, dv, templates_count, D = 24, 12, 32, 8, 768
    N, M = (heads + kv_heads) * dq + kv_heads * dv + heads * templates_count, boards * 70
    generator = torch.Generator().manual_seed(dq * 1000 + boards)
    x = torch.randint(-127, 128, (M, D), generator=generator, dtype=torch.int8).cuda()
    weight = torch.randint(-127, 128, (N, D), generator=generator, dtype=torch.int8).cuda()
    x_scale = (torch.rand(M, generator=generator) / 100 + 1e-3).cuda()
    weight_scale = (torch.rand(N, generator=generator) / 100 + 1e-3).cuda()
    bias = torch.randn(N, generator=generator).half().cuda()
    q_gain, k_gain = (1 + torch.randn(2, dq, generator=generator) / 10).half().cuda()
    paired = ops.pair_templates((torch.randn(8, 64, 64, generator=generator) / 2).half().cuda())
    plain = ops.int8_linear(x, x_scale, weight, weight_scale, bias, None, False, "projection")
    fused = torch.empty(M, N, dtype=torch.float16, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    pointer = lambda t: ctypes.c_void_p(t.data_ptr())
    lib.fry_int8_linear_qk_norm(pointer(x), pointer(x_scale), pointer(weight), pointer(weight_scale), pointer(bias), pointer(q_gain),
                                pointer(k_gain), 1e-5, pointer(fused), M, N, D, heads, kv_heads, dq, stream)
    qk = (heads + kv_heads) * dq
    assert torch.equal(fused[:, qk:], plain[:, qk:])
    assert not torch.equal(fused[:, :qk], plain[:, :qk])
    # each query and key head RMS-normalised with its gain, against fp32 to within fp16 rounding
    for first, count, gain in ((0, heads, q_gain), (heads * dq, kv_heads, k_gain)):
        rows = plain[:, first:first + count * dq].float().reshape(M, count, dq)
        normed = rows * torch.rsqrt(rows.square().mean(-1, keepdim=True) + 1e-5) * gain.float()
        assert torch.allclose(fused[:, first:first + count * dq].float().reshape(M, count, dq), normed, rtol=2e-3, atol=1e-3)
    expected = torch.empty(boards, 70, heads * dv, dtype=torch.float16, device="cuda")
    found = torch.empty_like(expected)
    lib.fry_template_attention(pointer(plain), pointer(paired), pointer(q_gain), pointer(k_gain), pointer(expected), boards, heads, kv_heads,
                               dq, dv, templates_count, 1e-5, stream)
    lib.fry_template_attention_normed(pointer(fused), pointer(paired), pointer(found), boards, heads, kv_heads, dq, dv, templates_count, stream)
    torch.cuda.synchronize()
    assert torch.isfinite(expected).all()
    assert torch.equal(found, expected)
