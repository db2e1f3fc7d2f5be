"""The microbench configuration's CPU checker, pinned without a GPU: its int32 sums against torch's integer matmul, its
checksums against those sums, its bf16 rounding against torch's fp32 -> bf16 conversion, and its attention against
torch's own scaled-dot-product attention in fp32."""
import numpy as np
import torch
import torch.nn.functional as F

from oracle import microbench as mb


def test_the_int32_sums_and_their_checksums_are_exact():
    x, weight, _, _ = mb.gemm_operands(300, 3072, 40, 1)
    acc = mb.int32_sums(x, weight)
    exact = torch.from_numpy(x).long() @ torch.from_numpy(weight).long().T
    assert np.array_equal(acc, exact.numpy())
    assert np.array_equal(mb.column_checksum(x, weight), exact.sum(0).numpy())
    assert np.array_equal(mb.row_checksum(x, weight), exact.sum(1).numpy())


def test_the_bf16_rounding_is_torchs():
    rng = np.random.default_rng(2)
    values = np.concatenate([rng.standard_normal(100000).astype(np.float32) * 10.0 ** rng.integers(-6, 6, 100000),
                             # exact ties between two bf16 neighbours, both parities
                             (np.arange(1, 2000, dtype=np.uint32) << 15 | np.uint32(0x3F800000)).view(np.float32)])
    found = mb.bf16_bits(values)
    expected = torch.from_numpy(values).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(found, expected)


def test_the_scaled_epilogue_meets_the_references_dequantised_criterion():
    # tests/test_int8.py:90's atol 1e-3, with rtol the bf16 output's own half step (2^-8 relative; the reference's
    # 2e-3 was set for fp16 outputs, whose half step is 2^-11)
    x, weight, x_scale, weight_scale = mb.gemm_operands(64, 768, 128, 3)
    out = mb.bf16_values(mb.scaled_bf16(mb.int32_sums(x, weight), x_scale, weight_scale))
    assert np.allclose(out, mb.dequantised(x, weight, x_scale, weight_scale), atol=1e-3, rtol=mb.BF16_RTOL)


def test_the_attention_is_torchs_scaled_dot_product_attention():
    q, k, v = mb.attention_operands(3, 4)
    split = lambda t: t.float().reshape(3, 64, 12, 64).transpose(1, 2)
    expected = F.scaled_dot_product_attention(split(q), split(k), split(v)).transpose(1, 2).reshape(3, 64, 768)
    assert torch.allclose(mb.attention_fp32(q, k, v), expected, atol=1e-5)
