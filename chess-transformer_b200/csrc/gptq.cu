// GPTQ on the device: `gptq` of engine/quantization.py:76-99 (Frantar et al. 2022), the rounding that turns a block's
// fp weights into its Int8Weights, in fp64 as the reference runs it.
//
//   H: inputs with a zero diagonal (no curvature: the down matmul's padding) get diagonal 1 and zero weights; then the
//      diagonal += 0.01 * its mean (gptq_diagonal_kernel, gptq_scale_kernel);
//   U: the inverse's upper Cholesky factor, H^-1 = U^T U (:87): H = L L^T (cholesky_*), X = L^-1 (lower_inverse_kernel),
//      H^-1 = X^T X (gram_lower_kernel), H^-1 = C C^T, U = C^T (read as C transposed, never formed);
//   scale a row = max(absmax, 1e-20) / 127;
//   columns in blocks of 128: each column rounded half to even and clamped to +-127, its error / U[i][i] spread over the
//      block's later columns (gptq_block_kernel, a thread a row), then the block's errors over every later column through
//      U (gptq_trailing_kernel).
//
// Every elementwise step is one IEEE fp64 operation in the reference's order (no contraction: explicit _rn intrinsics),
// so, the factorizations aside, a row's arithmetic is the reference's. The factorizations and products sum in their own
// orders; the reference keeps fp64 so that such last-bit differences round every weight alike (:78).
//
// This is offline work, run once per checkpoint: the kernels are plain SIMT fp64 and the Cholesky factorizations are
// right-looking, one launch pair a column.
#include "common.cuh"
#include "kernels.h"

namespace fry {

constexpr int kGptqColumns = 128;   // engine/quantization.py:45
constexpr double kDampening = 0.01; // engine/quantization.py:44
constexpr double kInt8Max = 127.0;  // engine/quantization.py:47
constexpr int kGptqMaxK = 4096, kGptqMaxN = 1 << 18;  // within the launch grids' bounds

GptqWorkspace::GptqWorkspace(size_t N, size_t K) {
    auto up = [](size_t bytes) { return (bytes + 255) / 256 * 256; };
    hessian = 0;
    inverse = hessian + up(K * K * sizeof(double));
    weight = inverse + up(K * K * sizeof(double));
    errors = weight + up(N * K * sizeof(double));
    scale = errors + up(N * kGptqColumns * sizeof(double));
    dead = scale + up(N * sizeof(double));
    total = dead + up(K * sizeof(int));
}

// One CTA of 1024 threads: flags the dead inputs and sets their diagonal to 1, then adds 0.01 of the diagonal's mean to
// it. The mean's sum runs in a fixed order: each thread's inputs in order, then a tree over the threads.
__global__ void __launch_bounds__(1024) gptq_diagonal_kernel(double* __restrict__ H, int* __restrict__ dead, int K) {
    __shared__ double partial[1024];
    double sum = 0.0;
    for (int k = threadIdx.x; k < K; k += blockDim.x) {
        double d = H[static_cast<size_t>(k) * K + k];
        dead[k] = d == 0.0;
        if (d == 0.0) {
            d = 1.0;
            H[static_cast<size_t>(k) * K + k] = 1.0;
        }
        sum = __dadd_rn(sum, d);
    }
    partial[threadIdx.x] = sum;
    __syncthreads();
    for (int width = blockDim.x / 2; width > 0; width >>= 1) {
        if (threadIdx.x < width) partial[threadIdx.x] = __dadd_rn(partial[threadIdx.x], partial[threadIdx.x + width]);
        __syncthreads();
    }
    const double damp = __dmul_rn(kDampening, __ddiv_rn(partial[0], static_cast<double>(K)));
    for (int k = threadIdx.x; k < K; k += blockDim.x) H[static_cast<size_t>(k) * K + k] = __dadd_rn(H[static_cast<size_t>(k) * K + k], damp);
}

// A warp a row: the dead inputs' weights zeroed, then scale = max(absmax, 1e-20) / 127 in fp64 and as fp32.
__global__ void gptq_scale_kernel(double* __restrict__ W, const int* __restrict__ dead, double* __restrict__ scale,
                                  float* __restrict__ out_scale, int N, int K) {
    const int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (r >= N) return;
    double* row = W + static_cast<size_t>(r) * K;
    double top = 0.0;
    for (int k = lane; k < K; k += 32) {
        double w = row[k];
        if (dead[k]) {
            w = 0.0;
            row[k] = 0.0;
        }
        top = fmax(top, fabs(w));
    }
#pragma unroll
    for (int offset = 16; offset > 0; offset >>= 1) top = fmax(top, __shfl_xor_sync(0xffffffffu, top, offset));
    if (lane == 0) {
        const double s = __ddiv_rn(fmax(top, 1e-20), kInt8Max);
        scale[r] = s;
        out_scale[r] = __double2float_rn(s);
    }
}

// Column j of a right-looking Cholesky factorization, A = L L^T in A's lower triangle: L[j][j] = sqrt(A[j][j]) and
// L[i][j] = A[i][j] / L[j][j] below it. One CTA. A pivot that is not positive is recorded (the factorization goes on
// with the NaN it makes; the host reports the failure).
__global__ void __launch_bounds__(1024) cholesky_column_kernel(double* __restrict__ A, int K, int j) {
    __shared__ double pivot;
    if (threadIdx.x == 0) {
        const double d = A[static_cast<size_t>(j) * K + j];
        if (!(d > 0.0)) record_error(kNotPositiveDefinite, j);
        pivot = __dsqrt_rn(d);
        A[static_cast<size_t>(j) * K + j] = pivot;
    }
    __syncthreads();
    for (int i = j + 1 + threadIdx.x; i < K; i += blockDim.x)
        A[static_cast<size_t>(i) * K + j] = __ddiv_rn(A[static_cast<size_t>(i) * K + j], pivot);
}

// The trailing update after column j: A[i][k] -= L[i][j] * L[k][j] for j < k <= i (lower triangle only).
__global__ void cholesky_update_kernel(double* __restrict__ A, int K, int j) {
    const int k = j + 1 + blockIdx.x * blockDim.x + threadIdx.x, i = j + 1 + blockIdx.y * blockDim.y + threadIdx.y;
    if (i >= K || k > i) return;
    const size_t at = static_cast<size_t>(i) * K + k;
    A[at] = __dsub_rn(A[at], __dmul_rn(A[static_cast<size_t>(i) * K + j], A[static_cast<size_t>(k) * K + j]));
}

// X = L^-1 for L lower triangular: column j solves L x = e_j by forward substitution, one thread a column.
__global__ void lower_inverse_kernel(const double* __restrict__ L, double* __restrict__ X, int K) {
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= K) return;
    for (int i = 0; i < j; ++i) X[static_cast<size_t>(i) * K + j] = 0.0;
    for (int i = j; i < K; ++i) {
        const double* l = L + static_cast<size_t>(i) * K;
        double s = i == j ? 1.0 : 0.0;
        for (int k = j; k < i; ++k) s = __dsub_rn(s, __dmul_rn(l[k], X[static_cast<size_t>(k) * K + j]));
        X[static_cast<size_t>(i) * K + j] = __ddiv_rn(s, l[i]);
    }
}

// G = X^T X for X lower triangular, the lower triangle: G[a][b] = sum over i >= a of X[i][a] X[i][b], b <= a.
__global__ void gram_lower_kernel(const double* __restrict__ X, double* __restrict__ G, int K) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x, a = blockIdx.y * blockDim.y + threadIdx.y;
    if (a >= K || b > a) return;
    double s = 0.0;
    for (int i = a; i < K; ++i) s = __fma_rn(X[static_cast<size_t>(i) * K + a], X[static_cast<size_t>(i) * K + b], s);
    G[static_cast<size_t>(a) * K + b] = s;
}

// GPTQ's column loop over the block [first, last), a thread a row (engine/quantization.py:92-97), with U[i][j] = C[j][i]:
// each column rounded half to even on the row's scale and clamped, its error (w - q * scale) / U[i][i] kept for the
// trailing update and spread over the block's columns from i on.
__global__ void gptq_block_kernel(double* __restrict__ W, const double* __restrict__ C, const double* __restrict__ scale,
                                  double* __restrict__ errors, int8_t* __restrict__ q, int N, int K, int first, int last) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= N) return;
    double* row = W + static_cast<size_t>(r) * K;
    const double s = scale[r];
    for (int i = first; i < last; ++i) {
        const double w = row[i];
        const double rounded = fmin(fmax(rint(__ddiv_rn(w, s)), -kInt8Max), kInt8Max);
        q[static_cast<size_t>(r) * K + i] = static_cast<int8_t>(static_cast<int>(rounded));
        const double e = __ddiv_rn(__dsub_rn(w, __dmul_rn(rounded, s)), C[static_cast<size_t>(i) * K + i]);
        errors[static_cast<size_t>(r) * kGptqColumns + (i - first)] = e;
        for (int j = i; j < last; ++j) row[j] = __dsub_rn(row[j], __dmul_rn(e, C[static_cast<size_t>(j) * K + i]));
    }
}

// The block's errors over every later column (engine/quantization.py:98): W[r][c] -= sum_i errors[r][i] U[first + i][c].
__global__ void gptq_trailing_kernel(double* __restrict__ W, const double* __restrict__ C, const double* __restrict__ errors, int N,
                                     int K, int first, int last) {
    const int c = last + blockIdx.x * blockDim.x + threadIdx.x, r = blockIdx.y * blockDim.y + threadIdx.y;
    if (c >= K || r >= N) return;
    const double* e = errors + static_cast<size_t>(r) * kGptqColumns;
    const double* u = C + static_cast<size_t>(c) * K + first;
    double s = 0.0;
    for (int i = 0; i < last - first; ++i) s = __fma_rn(e[i], u[i], s);
    const size_t at = static_cast<size_t>(r) * K + c;
    W[at] = __dsub_rn(W[at], s);
}

// H [K, K] += x^T x for x [rows, K] fp64 (the input sums of engine/quantization.py:103-119): a CTA a 32 x 32 tile of H
// on or below the diagonal, 16 x 16 threads of 2 x 2 outputs, rows in steps of 32 through shared memory. Each output sums
// its rows in order, is added to H, and is mirrored above the diagonal, so H stays exactly symmetric.
__global__ void __launch_bounds__(256) hessian_accumulate_kernel(const double* __restrict__ x, double* __restrict__ H, int rows, int K) {
    if (blockIdx.y < blockIdx.x) return;
    __shared__ double xa[32][33], xb[32][33];
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4, a0 = blockIdx.y * 32, b0 = blockIdx.x * 32;
    double acc[2][2] = {{0.0, 0.0}, {0.0, 0.0}};
    for (int r0 = 0; r0 < rows; r0 += 32) {
        for (int i = threadIdx.x; i < 32 * 32; i += blockDim.x) {
            const int rr = i >> 5, cc = i & 31, r = r0 + rr;
            xa[rr][cc] = r < rows && a0 + cc < K ? x[static_cast<size_t>(r) * K + a0 + cc] : 0.0;
            xb[rr][cc] = r < rows && b0 + cc < K ? x[static_cast<size_t>(r) * K + b0 + cc] : 0.0;
        }
        __syncthreads();
#pragma unroll 8
        for (int rr = 0; rr < 32; ++rr)
#pragma unroll
            for (int i = 0; i < 2; ++i)
#pragma unroll
                for (int j = 0; j < 2; ++j) acc[i][j] = __fma_rn(xa[rr][ty * 2 + i], xb[rr][tx * 2 + j], acc[i][j]);
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const int a = a0 + ty * 2 + i, b = b0 + tx * 2 + j;
            if (a >= K || b >= K) continue;
            const size_t at = static_cast<size_t>(a) * K + b;
            H[at] = __dadd_rn(H[at], acc[i][j]);
            if (a0 != b0) H[static_cast<size_t>(b) * K + a] = H[at];
        }
}

cudaError_t hessian_accumulate(const double* x, int rows, int K, double* H, cudaStream_t stream, std::string* error) {
    if (rows < 0 || K <= 0 || K > kGptqMaxK) {
        if (error) *error = "fry_hessian_accumulate takes rows >= 0 and 0 < K <= " + std::to_string(kGptqMaxK);
        return cudaErrorInvalidValue;
    }
    if (rows == 0) return cudaSuccess;
    const int tiles = (K + 31) / 32;
    hessian_accumulate_kernel<<<dim3(tiles, tiles), 256, 0, stream>>>(x, H, rows, K);
    return cudaGetLastError();
}

// A = L L^T in place (lower triangle), one column at a time.
cudaError_t cholesky_lower(double* A, int K, cudaStream_t stream) {
    const dim3 tile(32, 8);
    for (int j = 0; j < K; ++j) {
        cholesky_column_kernel<<<1, 1024, 0, stream>>>(A, K, j);
        const int rest = K - j - 1;
        if (rest > 0) cholesky_update_kernel<<<dim3((rest + 31) / 32, (rest + 7) / 8), tile, 0, stream>>>(A, K, j);
    }
    return cudaGetLastError();
}

cudaError_t gptq(const double* weight, const double* hessian, int N, int K, int8_t* q, float* out_scale, void* workspace,
                 size_t workspace_bytes, cudaStream_t stream, std::string* error) {
    if (N <= 0 || N > kGptqMaxN || K <= 0 || K > kGptqMaxK) {
        if (error) *error = "fry_gptq takes 0 < N <= " + std::to_string(kGptqMaxN) + " and 0 < K <= " + std::to_string(kGptqMaxK);
        return cudaErrorInvalidValue;
    }
    const GptqWorkspace layout(N, K);
    if (workspace_bytes < layout.total) {
        if (error) *error = "fry_gptq's workspace is smaller than fry_gptq_workspace_bytes";
        return cudaErrorInvalidValue;
    }
    uint8_t* base = static_cast<uint8_t*>(workspace);
    double* H = reinterpret_cast<double*>(base + layout.hessian);
    double* X = reinterpret_cast<double*>(base + layout.inverse);
    double* W = reinterpret_cast<double*>(base + layout.weight);
    double* E = reinterpret_cast<double*>(base + layout.errors);
    double* scale = reinterpret_cast<double*>(base + layout.scale);
    int* dead = reinterpret_cast<int*>(base + layout.dead);
    const size_t KK = static_cast<size_t>(K) * K, NK = static_cast<size_t>(N) * K;
    cudaError_t status;
    if ((status = cudaMemcpyAsync(H, hessian, KK * sizeof(double), cudaMemcpyDeviceToDevice, stream)) != cudaSuccess) return status;
    if ((status = cudaMemcpyAsync(W, weight, NK * sizeof(double), cudaMemcpyDeviceToDevice, stream)) != cudaSuccess) return status;
    gptq_diagonal_kernel<<<1, 1024, 0, stream>>>(H, dead, K);
    gptq_scale_kernel<<<(N * 32 + 255) / 256, 256, 0, stream>>>(W, dead, scale, out_scale, N, K);
    // U: H = L L^T, X = L^-1, H^-1 = X^T X = C C^T (into H's lower triangle)
    if ((status = cholesky_lower(H, K, stream)) != cudaSuccess) return status;
    lower_inverse_kernel<<<(K + 127) / 128, 128, 0, stream>>>(H, X, K);
    const dim3 tile(32, 8);
    gram_lower_kernel<<<dim3((K + 31) / 32, (K + 7) / 8), tile, 0, stream>>>(X, H, K);
    if ((status = cholesky_lower(H, K, stream)) != cudaSuccess) return status;
    for (int first = 0; first < K; first += kGptqColumns) {
        const int last = first + kGptqColumns < K ? first + kGptqColumns : K;
        gptq_block_kernel<<<(N + 127) / 128, 128, 0, stream>>>(W, H, scale, E, q, N, K, first, last);
        if (last < K) gptq_trailing_kernel<<<dim3((K - last + 31) / 32, (N + 7) / 8), tile, 0, stream>>>(W, H, E, N, K, first, last);
    }
    return cudaGetLastError();
}

}  // namespace fry
