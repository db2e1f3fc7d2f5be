"""The benchmark's isolated-kernel configuration on the GPU, through the C ABI (the fry:: ops): the int8 GEMM with the
per-row / per-column scale epilogue to bf16 at every (K, N) and M it names, and the attention at seq 64, head_dim 64,
12 heads, batch 64 and 1024.

The GEMM's int32 sums are exact: every row at M = 4096, and at the larger M sampled rows (the first and last of every
128-row block among them) plus each column's and each row's sum over the whole output against the exact int64
checksums. Its bf16 outputs equal the oracle's epilogue bit for bit and meet the reference's dequantised criterion
(tests/test_int8.py:59-90) with bf16's half step as the relative tolerance. The attention is within 1e-2 of fp32
(tests/test_attention_cuda.py:63-71)."""
import numpy as np
import pytest
import torch

from chess_transformer_b200 import ops
from chess_transformer_b200.build import build
from oracle import microbench as mb

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def built():
    build()


def sampled_rows(M: int, count: int, seed: int) -> np.ndarray:
    blocks = np.arange(0, M, 128)
    edges = np.concatenate([blocks, np.minimum(blocks + 127, M - 1)])
    rng = np.random.default_rng(seed)
    return np.unique(np.concatenate([edges[rng.choice(len(edges), min(len(edges), count // 2), replace=False)],
                                     rng.choice(M, count // 2, replace=False), [0, M - 1]]))


@pytest.mark.parametrize("M", mb.GEMM_ROWS)
@pytest.mark.parametrize("K, N", mb.GEMM_SHAPES)
def test_the_scaled_int8_gemm_is_exact_at_every_benchmark_shape(M, K, N):
    x, weight, x_scale, weight_scale = mb.gemm_operands(M, K, N, seed=M + K + N)
    xd, wd = torch.from_numpy(x).cuda(), torch.from_numpy(weight).cuda()
    sd, wsd = torch.from_numpy(x_scale).cuda(), torch.from_numpy(weight_scale).cuda()
    acc = ops.int8_matmul_i32(xd, wd)
    out = ops.int8_matmul_scaled_bf16(xd, sd, wd, wsd)
    assert out.dtype == torch.bfloat16 and out.shape == (M, N)
    rows = np.arange(M) if M <= 4096 else sampled_rows(M, 512, M)
    acc_rows = acc[torch.from_numpy(rows).cuda()].cpu().numpy()
    expected = mb.int32_sums(x[rows], weight)
    assert np.array_equal(acc_rows, expected)
    # every element's contribution, through the exact column and row checksums of the whole output
    assert np.array_equal(acc.long().sum(0).cpu().numpy(), mb.column_checksum(x, weight))
    assert np.array_equal(acc.long().sum(1).cpu().numpy(), mb.row_checksum(x, weight))
    out_rows = out[torch.from_numpy(rows).cuda()].view(torch.int16).cpu().numpy().view(np.uint16)
    assert np.array_equal(out_rows, mb.scaled_bf16(expected, x_scale[rows], weight_scale))
    values = mb.bf16_values(out_rows)
    assert np.allclose(values, mb.dequantised(x[rows], weight, x_scale[rows], weight_scale), atol=1e-3, rtol=mb.BF16_RTOL)


@pytest.mark.parametrize("M", [1, 70, 129])
def test_the_scaled_int8_gemm_takes_partial_row_blocks(M):
    x, weight, x_scale, weight_scale = mb.gemm_operands(M, 768, 2304, seed=M)
    out = ops.int8_matmul_scaled_bf16(torch.from_numpy(x).cuda(), torch.from_numpy(x_scale).cuda(), torch.from_numpy(weight).cuda(),
                                      torch.from_numpy(weight_scale).cuda())
    found = out.view(torch.int16).cpu().numpy().view(np.uint16)
    assert np.array_equal(found, mb.scaled_bf16(mb.int32_sums(x, weight), x_scale, weight_scale))


@pytest.mark.parametrize("B", mb.ATTENTION_BATCHES + (1, 3))
def test_the_attention_is_the_attention_in_fp32(B):
    q, k, v = mb.attention_operands(B, seed=B)
    out = ops.attention_bf16(q.cuda(), k.cuda(), v.cuda(), mb.ATTENTION_HEADS)
    expected = mb.attention_fp32(q, k, v)
    assert out.dtype == torch.bfloat16 and out.shape == expected.shape
    error = (out.float().cpu() - expected).abs()
    assert error.max() <= 1e-2, error.max()


def test_the_attention_refuses_other_shapes():
    from chess_transformer_b200.library import FryError
    q = torch.zeros(2, 70, 768, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(FryError, match="64 tokens"):
        ops.attention_bf16(q, q, q, 12)
    q = torch.zeros(2, 64, 768, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(FryError, match="64 wide"):
        ops.attention_bf16(q, q, q, 24)
