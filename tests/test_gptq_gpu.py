"""GPTQ on the device (fry_gptq, chess_transformer_b200.quantization.gptq) against the reference's own outputs, and
against the oracle at the sizes of Fry's matmuls."""
import numpy as np
import pytest
import torch

from chess_transformer_b200.build import build
from chess_transformer_b200.library import FryError, library
from chess_transformer_b200.quantization import gptq
from oracle import gptq as og
from tests.conftest import ROOT

pytestmark = pytest.mark.gpu

GOLDEN = ROOT / "tests" / "golden" / "gptq_golden.npz"


@pytest.fixture(scope="module", autouse=True)
def built():
    build()


@pytest.mark.parametrize("name", ["projection", "down"])
def test_device_gptq_is_the_references(name):
    golden = np.load(GOLDEN)
    integers, scale = gptq(torch.from_numpy(golden[f"{name}_weight"]).cuda(), torch.from_numpy(golden[f"{name}_hessian"]).cuda())
    assert integers.dtype == torch.int8 and scale.dtype == torch.float32
    assert np.array_equal(integers.cpu().numpy(), golden[f"{name}_int8"])
    assert np.array_equal(scale.cpu().numpy(), golden[f"{name}_scale"])


@pytest.mark.parametrize("N, K, dead", [(1984, 768, 0), (768, 1024, 32), (1296, 768, 0)])
def test_device_gptq_matches_the_oracle_at_frys_sizes(N, K, dead):
    # gate_up [1984, 768], down [768, 1024] with padding inputs of no curvature, projection [1296, 768] (dq 24); the Hessian
    # a sum of x^T x over 4096 seeded activations with per-input scales, as input_hessians builds it (:103-119)
    rng = np.random.default_rng(N + K)
    x = rng.standard_normal((4096, K)) * rng.uniform(0.2, 3.0, size=K)
    if dead:
        x[:, K - dead:] = 0
    hessian = x.T @ x
    weight = rng.standard_normal((N, K)) * 0.02
    expected, expected_scale = og.gptq(weight, hessian)
    integers, scale = gptq(torch.from_numpy(weight).cuda(), torch.from_numpy(hessian).cuda())
    found = integers.cpu().numpy()
    # the factorizations round in their own orders, last bits of fp64 apart: a weight whose quotient sits on a rounding
    # boundary to within that may round one step apart, nothing more
    assert np.array_equal(scale.cpu().numpy(), expected_scale)
    assert (found == expected).mean() >= 0.9999
    assert np.abs(found.astype(int) - expected.astype(int)).max() <= 1
    if dead:
        assert not found[:, K - dead:].any()


def test_a_hessian_that_is_not_positive_definite_raises_as_the_references_cholesky_does():
    lib = library()
    lib.device_status(clear=True)
    before = lib.device_status()
    hessian = -torch.eye(64, dtype=torch.float64)
    with pytest.raises(FryError, match="not positive definite"):
        gptq(torch.randn(16, 64, dtype=torch.float64).cuda(), hessian.cuda())
    assert lib.device_status() == before


def test_hessian_accumulate_sums_x_transpose_x_exactly_symmetric():
    lib = library()
    rng = np.random.default_rng(7)
    first, second = rng.standard_normal((700, 384)), rng.standard_normal((70, 384)) * 3
    hessian = torch.zeros(384, 384, dtype=torch.float64, device="cuda")
    for x in (first, second):
        xs = torch.from_numpy(x).cuda()
        lib.fry_hessian_accumulate(xs.data_ptr(), xs.shape[0], xs.shape[1], hessian.data_ptr(), torch.cuda.current_stream().cuda_stream)
    found = hessian.cpu().numpy()
    assert np.array_equal(found, found.T)
    assert np.allclose(found, first.T @ first + second.T @ second, rtol=1e-12, atol=1e-10)


def test_input_hessians_sum_each_matmuls_inputs():
    # engine/quantization.py:103-119 on a module with the reference's block structure: the sums of x^T x over the inputs
    # of each block's Q, gate_projection and down_projection
    from torch import nn
    from chess_transformer_b200.quantization import input_hessians

    class Block(nn.Module):
        def __init__(self):
            super().__init__()
            self.Q = nn.Linear(64, 64, bias=False)
            self.mlp = nn.Module()
            self.mlp.gate_projection, self.mlp.up_projection = nn.Linear(64, 96, bias=False), nn.Linear(64, 96, bias=False)
            self.mlp.down_projection = nn.Linear(96, 64, bias=False)

        def forward(self, x):
            x = x + self.Q(x).tanh()
            return x + self.mlp.down_projection(nn.functional.silu(self.mlp.gate_projection(x)) * self.mlp.up_projection(x))

    class Model(nn.Module):
        def __init__(self):
            super().__init__()
            self.embed = nn.Embedding(20, 64)
            self.encoder = nn.ModuleList([Block(), Block()])

        def forward(self, boards):
            x = self.embed(boards)
            for block in self.encoder:
                x = block(x)
            return x

    torch.manual_seed(3)
    model = Model().double().cuda()
    boards = torch.randint(0, 20, (300, 70), device="cuda")
    found = input_hessians(model, boards, batch=128)
    expected = [{} for _ in model.encoder]
    hooks = [layer.register_forward_pre_hook(lambda module, inputs, sums=sums, name=name: sums.__setitem__(
                 name, sums.get(name, 0) + inputs[0].reshape(-1, inputs[0].shape[-1]).t() @ inputs[0].reshape(-1, inputs[0].shape[-1])))
             for block, sums in zip(model.encoder, expected)
             for name, layer in (("projection", block.Q), ("gate_up", block.mlp.gate_projection), ("down", block.mlp.down_projection))]
    with torch.no_grad():
        for start in range(0, 300, 128):
            model(boards[start:start + 128])
    for hook in hooks:
        hook.remove()
    for got, want in zip(found, expected):
        for name in ("projection", "gate_up", "down"):
            assert torch.allclose(got[name], want[name], rtol=1e-11, atol=1e-9)


def test_int8_weights_from_the_references_sums_are_the_references():
    # engine/quantization.py:122-140 from block 0's raw sums: the projection's pair is the reference's to the bit, so its
    # int8 weights are too; the down's pair is rotated here in fp64 from the sums rounded to fp32, where the fixture's was
    # rounded to fp32 after rotation, so a weight on a rounding boundary may land one step apart
    from chess_transformer_b200.quantization import int8_weights_from_sums
    from oracle import model as om
    from tests.conftest import SMALL
    golden = np.load(GOLDEN)
    sums = {name: torch.from_numpy(golden[f"raw_{name}_hessian"]).double().cuda() for name in ("projection", "gate_up", "down")}
    weights = int8_weights_from_sums(om.seeded_state_dict(SMALL, 10), [sums], layers=[0])
    assert set(weights) == {0} and set(weights[0]) == {"projection", "gate_up", "down"}
    assert np.array_equal(weights[0]["projection"][0].cpu().numpy(), golden["projection_int8"])
    assert np.array_equal(weights[0]["projection"][1].cpu().numpy(), golden["projection_scale"])
    down = weights[0]["down"][0].cpu().numpy()
    assert (down == golden["down_int8"]).mean() >= 0.999 and np.abs(down.astype(int) - golden["down_int8"]).max() <= 1
    # the fixture's down weight was rounded to fp32 before its gptq; this one is the fp64 rotation's, so a row's absmax
    # (and scale) may sit one fp32 step apart
    assert np.allclose(weights[0]["down"][1].cpu().numpy(), golden["down_scale"], rtol=2e-7, atol=0)
