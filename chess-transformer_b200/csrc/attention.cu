// Template attention of a Fry block: `template_attention` (model/fused_blocks.py:35-171), the reference's CUDA
// variant being `template_attention_cuda` (model/attention_cuda.py:97-304).
//
// A position's 70 tokens (64 squares, 6 metadata) attend over all 70 keys. Per head: q and k RMS-normalised with gains
// and rounded to fp16; scores q.k * 1/sqrt(dq) in fp32, plus on the 64x64 square block the template bias
// fp16(sum_t c[i, h, t] * T[t, i, j]); softmax over the 70 keys; probabilities rounded to fp16 for the value product,
// whose fp32 sums are divided by the unrounded total. Grouped-query: head h reads key/value head h / (heads / kv_heads).
//
// One CTA per (position, group of up to 8 query heads), one warp per query head. The CTA stages its key/value heads'
// normalised keys and transposed values in shared memory; each warp walks its head's 5 row tiles of 16 queries with
// mma.sync m16n8k16 (fp16 in, fp32 accumulate): 70 x 80 scores and 16 x 32 outputs per tile are too small for
// tcgen05's 128-row tiles, and the bias is formed in registers from the templates (never materialised in HBM).
#include <cmath>
#include <string>

#include "common.cuh"
#include "kernels.h"

namespace fry {

constexpr int kAttnTokens = 70, kAttnSquares = 64, kAttnKeys = 80, kAttnDv = 32, kAttnTemplates = 8, kMaxHeadsPerCta = 8;

FRY_DEVICE void mma_f16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
FRY_DEVICE uint32_t pack_half2(float lo, float hi) {
    return static_cast<uint32_t>(f2h_bits(lo)) | (static_cast<uint32_t>(f2h_bits(hi)) << 16);
}
FRY_DEVICE float quad_sum(float v) {
    v += __shfl_xor_sync(0xffffffffu, v, 1);
    return v + __shfl_xor_sync(0xffffffffu, v, 2);
}
FRY_DEVICE float quad_max(float v) {
    v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 1));
    return fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 2));
}

// DQP: dq padded to the MMA depth (16 or 32). Shared: keys [kv][80][DQP + 8], values^T [kv][32][80 + 8] (fp16).
template <int DQP>
__global__ void __launch_bounds__(kMaxHeadsPerCta * 32) attention_kernel(const uint16_t* __restrict__ projected,
                                                                         const uint16_t* __restrict__ templates,
                                                                         const uint16_t* __restrict__ q_gain,
                                                                         const uint16_t* __restrict__ k_gain, uint16_t* __restrict__ out,
                                                                         int heads, int kv_heads, int dq, float eps, float scale) {
    constexpr int KROW = DQP + 8, VROW = kAttnKeys + 8, KS = DQP / 16;
    extern __shared__ __align__(16) uint16_t attn_smem[];
    const int heads_per_cta = blockDim.x / 32;
    const int group = heads / kv_heads;
    const int kv_per_cta = heads_per_cta / group;
    uint16_t* keys = attn_smem;                                  // [kv_per_cta][80][KROW]
    uint16_t* values = keys + kv_per_cta * kAttnKeys * KROW;     // [kv_per_cta][32][VROW]

    const int b = blockIdx.y, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
    const int width = (heads + kv_heads) * dq + kv_heads * kAttnDv + heads * kAttnTemplates;
    const int k_offset = heads * dq, v_offset = (heads + kv_heads) * dq, c_offset = v_offset + kv_heads * kAttnDv;
    const int first_kv = blockIdx.x * kv_per_cta;
    const uint16_t* board = projected + static_cast<size_t>(b) * kAttnTokens * width;

    // normalised keys, zero past dq and past the 70th key
    for (int item = tid; item < kv_per_cta * kAttnKeys; item += blockDim.x) {
        const int kv = item / kAttnKeys, key = item % kAttnKeys;
        uint16_t* row = keys + (kv * kAttnKeys + key) * KROW;
        float k[DQP];
        float squares = 0.0f;
#pragma unroll
        for (int i = 0; i < DQP; ++i) {
            k[i] = (key < kAttnTokens && i < dq) ? h2f_bits(board[key * width + k_offset + (first_kv + kv) * dq + i]) : 0.0f;
            squares = __fmaf_rn(k[i], k[i], squares);
        }
        const float inverse = rsqrtf(__fadd_rn(__fdiv_rn(squares, static_cast<float>(dq)), eps));
#pragma unroll
        for (int i = 0; i < DQP; ++i)
            row[i] = (key < kAttnTokens && i < dq) ? f2h_bits(__fmul_rn(__fmul_rn(k[i], inverse), h2f_bits(k_gain[i]))) : 0;
    }
    // values transposed: [kv][dv][key]
    for (int item = tid; item < kv_per_cta * kAttnKeys * (kAttnDv / 8); item += blockDim.x) {
        const int kv = item / (kAttnKeys * 4), rest = item % (kAttnKeys * 4), key = rest / 4, part = rest % 4;
        uint4 raw = make_uint4(0, 0, 0, 0);
        if (key < kAttnTokens)
            raw = *reinterpret_cast<const uint4*>(board + key * width + v_offset + (first_kv + kv) * kAttnDv + part * 8);
        const uint16_t* h = reinterpret_cast<const uint16_t*>(&raw);
#pragma unroll
        for (int i = 0; i < 8; ++i) values[(kv * kAttnDv + part * 8 + i) * VROW + key] = h[i];
    }
    __syncthreads();

    const int head = blockIdx.x * heads_per_cta + warp;
    const int kv = warp / group;
    const uint16_t* kv_keys = keys + kv * kAttnKeys * KROW;
    const uint16_t* kv_values = values + kv * kAttnDv * VROW;
    float qg[KS][2][2];
#pragma unroll
    for (int ks = 0; ks < KS; ++ks)
#pragma unroll
        for (int half = 0; half < 2; ++half)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int col = ks * 16 + half * 8 + 2 * t + e;
                qg[ks][half][e] = col < dq ? h2f_bits(q_gain[col]) : 0.0f;
            }

    for (int tile = 0; tile < 5; ++tile) {
        const int rows[2] = {tile * 16 + g, tile * 16 + g + 8};
        // queries: a[ks][0..3] per the m16n8k16 A layout, normalised per row (the row's dq values sit on the quad)
        float q[2][KS][2][2];
        float squares[2] = {0.0f, 0.0f};
#pragma unroll
        for (int r = 0; r < 2; ++r)
#pragma unroll
            for (int ks = 0; ks < KS; ++ks)
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    const int col = ks * 16 + half * 8 + 2 * t;
                    uint32_t raw = 0;
                    if (rows[r] < kAttnTokens && col < dq)
                        raw = *reinterpret_cast<const uint32_t*>(board + rows[r] * width + head * dq + col);
                    q[r][ks][half][0] = h2f_bits(static_cast<uint16_t>(raw & 0xffff));
                    q[r][ks][half][1] = h2f_bits(static_cast<uint16_t>(raw >> 16));
                    squares[r] = __fmaf_rn(q[r][ks][half][0], q[r][ks][half][0], squares[r]);
                    squares[r] = __fmaf_rn(q[r][ks][half][1], q[r][ks][half][1], squares[r]);
                }
        uint32_t a[KS][4];
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const float inverse = rsqrtf(__fadd_rn(__fdiv_rn(quad_sum(squares[r]), static_cast<float>(dq)), eps));
#pragma unroll
            for (int ks = 0; ks < KS; ++ks)
#pragma unroll
                for (int half = 0; half < 2; ++half)
                    a[ks][r + 2 * half] = pack_half2(__fmul_rn(__fmul_rn(q[r][ks][half][0], inverse), qg[ks][half][0]),
                                                     __fmul_rn(__fmul_rn(q[r][ks][half][1], inverse), qg[ks][half][1]));
        }
        // scores over 10 key tiles of 8
        float s[10][4];
#pragma unroll
        for (int j = 0; j < 10; ++j) {
            s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.0f;
            const uint16_t* key_row = kv_keys + (j * 8 + g) * KROW + 2 * t;
#pragma unroll
            for (int ks = 0; ks < KS; ++ks)
                mma_f16(s[j], a[ks][0], a[ks][1], a[ks][2], a[ks][3], *reinterpret_cast<const uint32_t*>(key_row + ks * 16),
                        *reinterpret_cast<const uint32_t*>(key_row + ks * 16 + 8));
        }
        // scale, template bias on the square block, mask past the 70th key
        float coefficient[2][kAttnTemplates];
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            if (rows[r] < kAttnSquares) {
                const uint4 raw = *reinterpret_cast<const uint4*>(board + rows[r] * width + c_offset + head * kAttnTemplates);
                const uint16_t* h = reinterpret_cast<const uint16_t*>(&raw);
#pragma unroll
                for (int i = 0; i < kAttnTemplates; ++i) coefficient[r][i] = h2f_bits(h[i]);
            }
        }
        float top[2] = {-INFINITY, -INFINITY};
#pragma unroll
        for (int j = 0; j < 10; ++j)
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                const int col = j * 8 + 2 * t;
                float bias[2] = {0.0f, 0.0f};
                if (rows[r] < kAttnSquares && col < kAttnSquares) {
#pragma unroll
                    for (int i = 0; i < kAttnTemplates; ++i) {
                        const uint32_t pair = *reinterpret_cast<const uint32_t*>(templates + (i * kAttnSquares + rows[r]) * kAttnSquares + col);
                        bias[0] = __fmaf_rn(coefficient[r][i], h2f_bits(static_cast<uint16_t>(pair & 0xffff)), bias[0]);
                        bias[1] = __fmaf_rn(coefficient[r][i], h2f_bits(static_cast<uint16_t>(pair >> 16)), bias[1]);
                    }
                    bias[0] = h2f_bits(f2h_bits(bias[0]));
                    bias[1] = h2f_bits(f2h_bits(bias[1]));
                }
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    float value = __fadd_rn(__fmul_rn(s[j][2 * r + e], scale), bias[e]);
                    if (col + e >= kAttnTokens) value = -INFINITY;
                    s[j][2 * r + e] = value;
                    top[r] = fmaxf(top[r], value);
                }
            }
        float total[2] = {0.0f, 0.0f};
#pragma unroll
        for (int r = 0; r < 2; ++r) top[r] = quad_max(top[r]);
#pragma unroll
        for (int j = 0; j < 10; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float p = ex2_approx(__fmul_rn(__fsub_rn(s[j][e], top[e >> 1]), 1.4426950408889634f));
                s[j][e] = p;
                total[e >> 1] = __fadd_rn(total[e >> 1], p);
            }
#pragma unroll
        for (int r = 0; r < 2; ++r) total[r] = quad_sum(total[r]);
        // out = P V over 5 key steps of 16
        float o[4][4];
#pragma unroll
        for (int n = 0; n < 4; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
#pragma unroll
        for (int kk = 0; kk < 5; ++kk) {
            const uint32_t p0 = pack_half2(s[2 * kk][0], s[2 * kk][1]), p1 = pack_half2(s[2 * kk][2], s[2 * kk][3]);
            const uint32_t p2 = pack_half2(s[2 * kk + 1][0], s[2 * kk + 1][1]), p3 = pack_half2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
            for (int n = 0; n < 4; ++n) {
                const uint16_t* value_row = kv_values + (n * 8 + g) * VROW + kk * 16 + 2 * t;
                mma_f16(o[n], p0, p1, p2, p3, *reinterpret_cast<const uint32_t*>(value_row), *reinterpret_cast<const uint32_t*>(value_row + 8));
            }
        }
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            if (rows[r] >= kAttnTokens) continue;
            uint16_t* to = out + (static_cast<size_t>(b) * kAttnTokens + rows[r]) * (heads * kAttnDv) + head * kAttnDv + 2 * t;
#pragma unroll
            for (int n = 0; n < 4; ++n)
                *reinterpret_cast<uint32_t*>(to + n * 8) =
                    pack_half2(__fdiv_rn(o[n][2 * r], total[r]), __fdiv_rn(o[n][2 * r + 1], total[r]));
        }
    }
}

cudaError_t template_attention(const uint16_t* projected, const uint16_t* templates, const uint16_t* q_gain, const uint16_t* k_gain,
                               uint16_t* out, int B, int heads, int kv_heads, int dq, int dv, int templates_count, float eps,
                               cudaStream_t stream, std::string* error) {
    if (B <= 0) return cudaSuccess;
    const int group = kv_heads > 0 ? heads / kv_heads : 0;
    const int per_cta = heads < kMaxHeadsPerCta ? heads : kMaxHeadsPerCta;
    const int width = (heads + kv_heads) * dq + kv_heads * dv + heads * templates_count;
    if (dv != kAttnDv || templates_count != kAttnTemplates || dq < 1 || dq > 32 || dq % 2 || kv_heads <= 0 || heads % kv_heads ||
        heads % per_cta || per_cta % group || ((heads + kv_heads) * dq) % 8 || width % 8) {
        if (error)
            *error = "template attention takes dv 32, 8 templates, an even dq up to 32, and head groups that fit 8 heads a CTA; got heads " +
                     std::to_string(heads) + ", kv heads " + std::to_string(kv_heads) + ", dq " + std::to_string(dq) + ", dv " +
                     std::to_string(dv);
        return cudaErrorInvalidValue;
    }
    const int kv_per_cta = per_cta / group;
    const float scale = static_cast<float>(1.0 / std::sqrt(static_cast<double>(dq)));  // 1 / math.sqrt(dq), rounded once to fp32
    const dim3 grid(heads / per_cta, B);
    if (dq <= 16) {
        const size_t bytes = (kv_per_cta * kAttnKeys * (16 + 8) + kv_per_cta * kAttnDv * (kAttnKeys + 8)) * sizeof(uint16_t);
        attention_kernel<16><<<grid, per_cta * 32, bytes, stream>>>(projected, templates, q_gain, k_gain, out, heads, kv_heads, dq, eps,
                                                                    scale);
    } else {
        const size_t bytes = (kv_per_cta * kAttnKeys * (32 + 8) + kv_per_cta * kAttnDv * (kAttnKeys + 8)) * sizeof(uint16_t);
        attention_kernel<32><<<grid, per_cta * 32, bytes, stream>>>(projected, templates, q_gain, k_gain, out, heads, kv_heads, dq, eps,
                                                                    scale);
    }
    return cudaGetLastError();
}

}  // namespace fry
