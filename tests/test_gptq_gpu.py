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
