"""The reference's GPTQ rounding restated in numpy on the CPU. TEST INFRASTRUCTURE ONLY.

`gptq(weight, hessian)` follows engine/quantization.py:76-99 (GPTQ, Frantar et al. 2022) step by step, in fp64:

- inputs with no curvature (a zero Hessian diagonal, the down matmul's padding) get diagonal 1 and zero weights
  (:80-84);
- the diagonal is dampened by 0.01 of its mean (:85, DAMPENING :44);
- the inverse Hessian's upper Cholesky factor U, H^-1 = U^T U (:87), by Cholesky, inverse and Cholesky again;
- a scale a row, absmax / 127 (:88, INT8_MAX :47);
- columns in blocks of 128 (GPTQ_COLUMNS :45): each column rounded half to even and clamped to +-127, its error divided
  by U's diagonal and spread over the block's later columns (:92-97), then the block's errors over every later column
  through U (:98).

Each elementwise step is one IEEE fp64 operation, as the reference's tensor ops are; the factorizations and the matrix
product round in LAPACK's and BLAS's orders, which may differ from the reference's in the last bits of fp64 (the
reference chose fp64 so that such differences round every weight alike, :78).
"""
import numpy as np

DAMPENING = 0.01      # engine/quantization.py:44
GPTQ_COLUMNS = 128    # engine/quantization.py:45
INT8_MAX = 127        # engine/quantization.py:47


def gptq(weight: np.ndarray, hessian: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """weight [N, K], hessian [K, K] (any float dtype, taken as fp64) -> (int8 [N, K], fp32 scale [N])."""
    weight = np.array(weight, dtype=np.float64)
    hessian = np.array(hessian, dtype=np.float64)
    K = weight.shape[1]
    diagonal = np.diagonal(hessian).copy()
    dead = diagonal == 0
    diagonal[dead] = 1
    weight[:, dead] = 0
    diagonal += DAMPENING * diagonal.mean()
    hessian[np.arange(K), np.arange(K)] = diagonal
    lower = np.linalg.cholesky(hessian)
    inverse_lower = np.linalg.inv(lower)
    inverse = np.linalg.cholesky(inverse_lower.T @ inverse_lower).T  # upper: H^-1 = U^T U
    scale = np.maximum(np.abs(weight).max(axis=1), 1e-20) / INT8_MAX
    integers = np.zeros_like(weight)
    for first in range(0, K, GPTQ_COLUMNS):
        last = min(first + GPTQ_COLUMNS, K)
        columns, block_inverse = weight[:, first:last].copy(), inverse[first:last, first:last]
        errors = np.zeros_like(columns)
        for i in range(last - first):
            rounded = np.clip(np.rint(columns[:, i] / scale), -INT8_MAX, INT8_MAX)
            integers[:, first + i] = rounded
            errors[:, i] = (columns[:, i] - rounded * scale) / block_inverse[i, i]
            columns[:, i:] -= errors[:, i, None] * block_inverse[i, i:]
        weight[:, last:] -= errors @ inverse[first:last, last:]
    return integers.astype(np.int8), scale.astype(np.float32)
