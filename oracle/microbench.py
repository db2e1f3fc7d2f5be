"""The isolated-kernel configuration's operands and answers on the CPU. TEST INFRASTRUCTURE ONLY.

The benchmark's microbench configuration runs two kernels outside Fry's own shapes: int8 x int8 -> int32 GEMMs with a
per-row / per-column scale epilogue to bf16, at (K, N) in {(768, 2304), (768, 768), (768, 3072), (3072, 768)} and M in
{4096, 16384, 65536}; and attention with seq 64, head_dim 64, 12 heads, batch 64 and 1024, on bf16 q/k/v. The
reference has no op of either shape, so the checker here is the plain arithmetic the reference's own tests check
kernels of the same families against:

- the int8 GEMM against the dequantised matmul in fp64, atol 1e-3 / rtol 2e-3 (tests/test_int8.py:59-90), the rtol
  widened to bf16's half step for the bf16 output; its int32 sums exactly (the int8 products summed in fp64 are exact
  below 2^53); its bf16 outputs bit for bit against the epilogue's own op order;
- the attention against fp32 torch, atol 1e-2 (tests/test_attention_cuda.py:51-71).

The operands follow the configuration's text: int8 uniform in [-127, 127], scales uniform in [1e-3, 1e-2], attention
inputs N(0, 1) rounded to bf16, all seeded.
"""
import numpy as np
import torch

GEMM_SHAPES = ((768, 2304), (768, 768), (768, 3072), (3072, 768))  # (K, N)
GEMM_ROWS = (4096, 16384, 65536)                                     # M
ATTENTION_BATCHES = (64, 1024)
ATTENTION_HEADS, ATTENTION_SEQ, ATTENTION_DIM = 12, 64, 64
# the dequantised criterion's relative tolerance for a bf16 output: its rounding alone is up to half a step, 2^-8 of
# the value (the reference's rtol 2e-3, tests/test_int8.py:90, was set for fp16 outputs), plus fp32's own slack
BF16_RTOL = 2.0 ** -8 + 1e-5


def gemm_operands(M: int, K: int, N: int, seed: int) -> tuple[np.ndarray, np.ndarray, np.ndarray, np.ndarray]:
    """x int8 [M, K], weight int8 [N, K], x_scale fp32 [M], weight_scale fp32 [N]."""
    rng = np.random.default_rng(seed)
    x = rng.integers(-127, 128, size=(M, K), dtype=np.int8)
    weight = rng.integers(-127, 128, size=(N, K), dtype=np.int8)
    x_scale = rng.uniform(1e-3, 1e-2, size=M).astype(np.float32)
    weight_scale = rng.uniform(1e-3, 1e-2, size=N).astype(np.float32)
    return x, weight, x_scale, weight_scale


def int32_sums(x: np.ndarray, weight: np.ndarray) -> np.ndarray:
    """acc = x . weight^T, exactly (fp64 holds every partial sum of K <= 2^20 int8 products exactly)."""
    return (x.astype(np.float64) @ weight.astype(np.float64).T).astype(np.int32)


def column_checksum(x: np.ndarray, weight: np.ndarray) -> np.ndarray:
    """sum over rows of acc, per column, exactly in int64: (sum_m x[m]) . weight^T."""
    return weight.astype(np.int64) @ x.sum(axis=0, dtype=np.int64)


def row_checksum(x: np.ndarray, weight: np.ndarray, chunk: int = 8192) -> np.ndarray:
    """sum over columns of acc, per row, exactly in int64: x . (sum_n weight[n]), a chunk of rows at a time."""
    totals = weight.sum(axis=0, dtype=np.int64)
    return np.concatenate([x[start:start + chunk].astype(np.int64) @ totals for start in range(0, len(x), chunk)])


def bf16_bits(values: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 (as uint16 bits), rounded to nearest with ties to even (finite inputs)."""
    bits = values.astype(np.float32).view(np.uint32).astype(np.uint64)
    rounded = (bits + 0x7FFF + ((bits >> 16) & 1)) >> 16
    return rounded.astype(np.uint16)


def bf16_values(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


def scaled_bf16(acc: np.ndarray, x_scale: np.ndarray, weight_scale: np.ndarray) -> np.ndarray:
    """The epilogue's bits: bf16((fp32(acc) * x_scale[m]) * weight_scale[n]), each product rounded to fp32."""
    product = (acc.astype(np.float32) * x_scale[:, None]).astype(np.float32)
    return bf16_bits((product * weight_scale[None, :]).astype(np.float32))


def dequantised(x: np.ndarray, weight: np.ndarray, x_scale: np.ndarray, weight_scale: np.ndarray) -> np.ndarray:
    """The dequantised matmul in fp64, the reference test's expectation (tests/test_int8.py:54-55,75)."""
    return (x.astype(np.float64) * x_scale.astype(np.float64)[:, None]) @ (weight.astype(np.float64) * weight_scale.astype(np.float64)[:, None]).T


def attention_operands(B: int, seed: int) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """q, k, v bf16 [B, 64, 12 * 64], N(0, 1)."""
    generator = torch.Generator().manual_seed(seed)
    shape = (B, ATTENTION_SEQ, ATTENTION_HEADS * ATTENTION_DIM)
    return tuple(torch.randn(shape, generator=generator).to(torch.bfloat16) for _ in range(3))


def attention_fp32(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, heads: int = ATTENTION_HEADS) -> torch.Tensor:
    """softmax(q k^T / sqrt(d)) v per sequence and head in fp32, [B, S, heads * d] in and out."""
    B, S, width = q.shape
    d = width // heads
    split = lambda t: t.float().reshape(B, S, heads, d).transpose(1, 2)
    scores = split(q) @ split(k).transpose(-2, -1) / d ** 0.5
    return (torch.softmax(scores, dim=-1) @ split(v)).transpose(1, 2).reshape(B, S, width)
