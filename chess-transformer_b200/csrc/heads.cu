// The heads after the last block: stream [B, 70, d] fp16 -> answer rows [B, 1969] fp32 (1968 move logits, then the
// expected score). The reference's B200 path is the torch one of `FusedTransformer.forward` (model/fused_blocks.py:863-874)
// with the weights folded by `head_weights` (:815-824), and `answer_rows` (engine/inference.py:19-23):
//
//   y = RMSNorm(x) in fp16;  a = y . A + a_bias (A = W_f^T W_t / sqrt d in fp16, fp32 accumulate);
//   narrow = y . N^T + n_bias (fp32): s (1), the 4 promotion logits, the 16 board-down units;
//   logit[f, t] = a_f . y_t + s_f, gathered to the 1968 moves, promotions plus their piece's logit at the landing square;
//   value = Linear(GELU(Linear(GELU(board-down) flattened))) ; score = softmax(value) . bin centres.
//
// Kernels: rms_norm (rows.cu), the tcgen05 f16 GEMM for a (gemm.cu), narrow_kernel, policy_kernel (per board: the 64x64
// logits from split-fp16 mma.sync, a = hi + lo / 2048 so the products stay fp32-exact), eval_linear_kernel (the eval head's
// two layers over all boards), expected_score_kernel (softmax times the bin centres). fp32 arithmetic throughout, where the
// reference uses tf32 matmuls.
#include <string>

#include "common.cuh"
#include "kernels.h"
#include "moves.h"

namespace fry {

constexpr int kHeadTokens = 70, kHeadSquares = 64, kNarrow = 21, kNarrowStride = 24, kDown = 16, kMoves = 1968;
constexpr float kLoScale = 2048.0f;

size_t heads_workspace_bytes(int B, int D) {
    const size_t M = static_cast<size_t>(B) * kHeadTokens;
    auto up = [](size_t bytes) { return (bytes + 255) / 256 * 256; };
    // y, a, narrow, then the eval head's hidden units [B, D] and value logits [B, up to 256 bins]
    return up(M * D * 2) + up(M * D * 4) + up(M * kNarrowStride * 4) + up(static_cast<size_t>(B) * (D + 256) * 4);
}

// narrow[m, 0..20] = y[m] . N^T + n_bias, 8 warps a CTA, the weights staged in shared memory.
__global__ void __launch_bounds__(256) narrow_kernel(const uint16_t* __restrict__ y, const float* __restrict__ weight,
                                                     const float* __restrict__ bias, float* __restrict__ narrow, int M, int D) {
    extern __shared__ float narrow_weights[];  // [21][D]
    for (int i = threadIdx.x; i < kNarrow * D; i += blockDim.x) narrow_weights[i] = weight[i];
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int m = blockIdx.x * 8 + warp; m < M; m += gridDim.x * 8) {
        float acc[kNarrow];
#pragma unroll
        for (int j = 0; j < kNarrow; ++j) acc[j] = 0.0f;
        for (int k = lane; k < D; k += 32) {
            const float v = h2f_bits(y[static_cast<size_t>(m) * D + k]);
#pragma unroll
            for (int j = 0; j < kNarrow; ++j) acc[j] = __fmaf_rn(v, narrow_weights[j * D + k], acc[j]);
        }
#pragma unroll
        for (int j = 0; j < kNarrow; ++j) {
            const float total = warp_sum(acc[j]);
            if (lane == j) narrow[static_cast<size_t>(m) * kNarrowStride + j] = __fadd_rn(total, bias[j]);
        }
    }
}

FRY_DEVICE void mma_f16_heads(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

FRY_DEVICE void split_pair(float2 v, uint32_t& hi, uint32_t& lo) {
    const __half h0 = __float2half_rn(v.x), h1 = __float2half_rn(v.y);
    const __half l0 = __float2half_rn(__fmul_rn(__fsub_rn(v.x, __half2float(h0)), kLoScale));
    const __half l1 = __float2half_rn(__fmul_rn(__fsub_rn(v.y, __half2float(h1)), kLoScale));
    hi = static_cast<uint32_t>(__half_as_ushort(h0)) | (static_cast<uint32_t>(__half_as_ushort(h1)) << 16);
    lo = static_cast<uint32_t>(__half_as_ushort(l0)) | (static_cast<uint32_t>(__half_as_ushort(l1)) << 16);
}

// One CTA (8 warps) per board: L = a_sq . y_sq^T (64 x 64), then the 1968 move logits.
__global__ void __launch_bounds__(256) policy_kernel(const float* __restrict__ a, const uint16_t* __restrict__ y,
                                                     const float* __restrict__ narrow, float* __restrict__ rows, int D) {
    __shared__ float logits[kHeadSquares][kHeadSquares + 1];
    const int b = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int m_tile = warp >> 1, n_first = (warp & 1) * 4;
    const size_t board = static_cast<size_t>(b) * kHeadTokens;
    float hi[4][4], lo[4][4];
#pragma unroll
    for (int n = 0; n < 4; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) hi[n][e] = lo[n][e] = 0.0f;
    const float* a_rows[2] = {a + (board + m_tile * 16 + g) * D, a + (board + m_tile * 16 + g + 8) * D};
    for (int k = 0; k < D; k += 16) {
        uint32_t ah[4], al[4];
        split_pair(*reinterpret_cast<const float2*>(a_rows[0] + k + 2 * t), ah[0], al[0]);
        split_pair(*reinterpret_cast<const float2*>(a_rows[1] + k + 2 * t), ah[1], al[1]);
        split_pair(*reinterpret_cast<const float2*>(a_rows[0] + k + 8 + 2 * t), ah[2], al[2]);
        split_pair(*reinterpret_cast<const float2*>(a_rows[1] + k + 8 + 2 * t), ah[3], al[3]);
#pragma unroll
        for (int n = 0; n < 4; ++n) {
            const uint16_t* y_row = y + (board + (n_first + n) * 8 + g) * D + k + 2 * t;
            const uint32_t b0 = *reinterpret_cast<const uint32_t*>(y_row), b1 = *reinterpret_cast<const uint32_t*>(y_row + 8);
            mma_f16_heads(hi[n], ah, b0, b1);
            mma_f16_heads(lo[n], al, b0, b1);
        }
    }
#pragma unroll
    for (int n = 0; n < 4; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int row = m_tile * 16 + g + (e >> 1) * 8, col = (n_first + n) * 8 + 2 * t + (e & 1);
            logits[row][col] = __fadd_rn(hi[n][e], __fdiv_rn(lo[n][e], kLoScale));
        }
    __syncthreads();
    const float* board_narrow = narrow + board * kNarrowStride;
    for (int m = threadIdx.x; m < kMoves; m += blockDim.x) {
        const int pair = kMovePairs[m], from = pair >> 6, to = pair & 63;
        float logit = __fadd_rn(logits[from][to], board_narrow[from * kNarrowStride]);
        const int promotion = kMovePromotion[m];
        if (promotion >= 0) logit = __fadd_rn(logit, board_narrow[to * kNarrowStride + 1 + promotion]);
        rows[static_cast<size_t>(b) * (kMoves + 1) + m] = logit;
    }
}

FRY_DEVICE float gelu(float x) { return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f)); }

// The eval head's two layers as one tiled fp32 kernel over all boards, 32 boards x 32 outputs a CTA, 2 x 2 a thread:
//   FROM_NARROW: out[b, u] = GELU(bias[u] + sum_i W[u, i] * GELU(narrow[b, i / 16, 5 + i % 16]))   (K = 70 x 16)
//   otherwise:   out[b, u] = bias[u] + sum_i W[u, i] * x[b, i]                                    (K = d)
template <bool FROM_NARROW>
__global__ void __launch_bounds__(256) eval_linear_kernel(const float* __restrict__ x, const float* __restrict__ weight,
                                                          const float* __restrict__ bias, float* __restrict__ out, int B, int K, int N) {
    constexpr int TB = 32, TU = 32, TK = 32;
    __shared__ float xs[TK][TB + 1];
    __shared__ float ws[TK][TU + 1];
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int b0 = blockIdx.y * TB, u0 = blockIdx.x * TU;
    float acc[2][2] = {};
    for (int k0 = 0; k0 < K; k0 += TK) {
        for (int i = threadIdx.x; i < TK * TB; i += 256) {
            const int kk = i % TK, bb = i / TK, input = k0 + kk, board = b0 + bb;
            float v = 0.0f;
            if (board < B && input < K) {
                if constexpr (FROM_NARROW)
                    v = gelu(x[(static_cast<size_t>(board) * kHeadTokens + input / kDown) * kNarrowStride + 5 + input % kDown]);
                else
                    v = x[static_cast<size_t>(board) * K + input];
            }
            xs[kk][bb] = v;
        }
        for (int i = threadIdx.x; i < TK * TU; i += 256) {
            const int kk = i % TK, uu = i / TK, input = k0 + kk, unit = u0 + uu;
            ws[kk][uu] = (unit < N && input < K) ? weight[static_cast<size_t>(unit) * K + input] : 0.0f;
        }
        __syncthreads();
#pragma unroll 8
        for (int kk = 0; kk < TK; ++kk)
#pragma unroll
            for (int i = 0; i < 2; ++i)
#pragma unroll
                for (int j = 0; j < 2; ++j) acc[i][j] = __fmaf_rn(xs[kk][ty * 2 + i], ws[kk][tx * 2 + j], acc[i][j]);
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const int board = b0 + ty * 2 + i, unit = u0 + tx * 2 + j;
            if (board < B && unit < N) {
                const float value = __fadd_rn(acc[i][j], bias[unit]);
                out[static_cast<size_t>(board) * N + unit] = FROM_NARROW ? gelu(value) : value;
            }
        }
}

// One warp per board: the softmax of its value logits times the bin centres (2i + 1) / 2bins, into the row's last column.
__global__ void __launch_bounds__(256) expected_score_kernel(const float* __restrict__ logits, float* __restrict__ rows, int B, int bins) {
    const int b = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (b >= B) return;
    const float* row = logits + static_cast<size_t>(b) * bins;
    float top = -INFINITY;
    for (int bin = lane; bin < bins; bin += 32) top = fmaxf(top, row[bin]);
    top = warp_max(top);
    float total = 0.0f, weighted = 0.0f;
    for (int bin = lane; bin < bins; bin += 32) {
        const float p = expf(__fsub_rn(row[bin], top));
        total = __fadd_rn(total, p);
        weighted = __fmaf_rn(p, __fdiv_rn(static_cast<float>(2 * bin + 1), static_cast<float>(2 * bins)), weighted);
    }
    total = warp_sum(total);
    weighted = warp_sum(weighted);
    if (lane == 0) rows[static_cast<size_t>(b) * (kMoves + 1) + kMoves] = __fdiv_rn(weighted, total);
}

cudaError_t heads(const uint16_t* stream_x, const HeadWeights& w, float eps, float* rows, void* workspace, size_t workspace_bytes, int B,
                  int D, cudaStream_t stream, std::string* error) {
    if (B <= 0) return cudaSuccess;
    if (workspace_bytes < heads_workspace_bytes(B, D)) {
        if (error) *error = "the heads' workspace is smaller than fry_heads_workspace_bytes";
        return cudaErrorInvalidValue;
    }
    if (D % 16 != 0 || D > 1024 || w.bins < 2 || w.bins > 256) {
        if (error) *error = "the heads take d_model a multiple of 16 up to 1024 and 2 to 256 value bins";
        return cudaErrorInvalidValue;
    }
    const int M = B * kHeadTokens;
    auto up = [](size_t bytes) { return (bytes + 255) / 256 * 256; };
    uint8_t* base = static_cast<uint8_t*>(workspace);
    uint16_t* y = reinterpret_cast<uint16_t*>(base);
    float* a = reinterpret_cast<float*>(base + up(static_cast<size_t>(M) * D * 2));
    float* narrow = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(a) + up(static_cast<size_t>(M) * D * 4));
    float* hidden = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(narrow) + up(static_cast<size_t>(M) * kNarrowStride * 4));

    cudaError_t status = rms_norm_f16(stream_x, w.ln_gain, eps, y, M, D, stream);
    if (status != cudaSuccess) return status;
    GemmArgs args;
    args.bias_f32 = w.a_bias;
    args.out = a;
    status = gemm(1, kEpiLinearF32, y, w.a_weight, args, M, D, D, stream, error);
    if (status != cudaSuccess) return status;
    const size_t narrow_smem = static_cast<size_t>(kNarrow) * D * sizeof(float);
    status = ensure_smem(reinterpret_cast<const void*>(narrow_kernel), static_cast<int>(narrow_smem));
    if (status != cudaSuccess) return status;
    const int narrow_blocks = (M + 31) / 32 < 148 * 4 ? (M + 31) / 32 : 148 * 4;
    narrow_kernel<<<narrow_blocks, 256, narrow_smem, stream>>>(y, w.narrow_weight, w.narrow_bias, narrow, M, D);
    policy_kernel<<<B, 256, 0, stream>>>(a, y, narrow, rows, D);
    float* value_logits = hidden + static_cast<size_t>(B) * D;
    eval_linear_kernel<true><<<dim3((D + 31) / 32, (B + 31) / 32), 256, 0, stream>>>(narrow, w.hidden_weight, w.hidden_bias, hidden, B,
                                                                                      kHeadTokens * kDown, D);
    eval_linear_kernel<false><<<dim3((w.bins + 31) / 32, (B + 31) / 32), 256, 0, stream>>>(hidden, w.out_weight, w.out_bias, value_logits, B,
                                                                                          D, w.bins);
    expected_score_kernel<<<(B + 7) / 8, 256, 0, stream>>>(value_logits, rows, B, w.bins);
    return cudaGetLastError();
}

}  // namespace fry
