// Template attention of a Fry block: `template_attention` (model/fused_blocks.py:35-171), the reference's CUDA
// variant being `template_attention_cuda` (model/attention_cuda.py:97-304).
//
// A position's 70 tokens (64 squares, 6 metadata) attend over all 70 keys. Per head: q and k RMS-normalised with gains
// and rounded to fp16; scores q.k * 1/sqrt(dq) in fp32, plus on the 64x64 square block the template bias
// fp16(sum_t c[i, h, t] * T[t, i, j]); softmax over the 70 keys; probabilities rounded to fp16 for the value product,
// whose fp32 sums are divided by the unrounded total. Grouped-query: head h reads key/value head h / (heads / kv_heads).
//
// One CTA per (position, group of up to 8 query heads), one warp per query head, in 5 phases: the 4 slabs of 16 square
// rows, then the metadata rows (at small batches one CTA per phase, so more SMs share a position). The CTA stages its key/value heads' normalised keys and raw values in shared memory.
// Before a square slab, the warps form its template bias for all the CTA's heads with mma.sync: for a pair of squares
// (i0, i1), A = the 8 heads' coefficients block-diagonally over (i0's 8 templates | i1's 8 templates) and B = the pair's
// templates, paired per key as [square][key][template] (fry_pair_templates, as the reference pairs them,
// model/attention_cuda.py:412-434), so one m16n8k16 gives 8 heads x 2 squares x 8 keys of bias. Each warp then takes
// its head's 16 rows: scores over 9 key tiles, bias added from the slab, softmax in registers (paired fp32 arithmetic,
// f32x2), P.V with the values' B fragments read by ldmatrix.trans. The next slab is formed in the same buffer once every
// warp has added the current one, while the exponentials run. 70 x 80 scores and 16 x 32 outputs per tile are too small
// for tcgen05's 128-row tiles; the legacy mma.sync keeps them in registers.
#include <cmath>
#include <string>
#include <type_traits>

#include "common.cuh"
#include "kernels.h"

namespace fry {

constexpr int kAttnTokens = 70, kAttnSquares = 64, kAttnKeys = 80, kAttnDv = 32, kAttnTemplates = 8, kMaxHeadsPerCta = 8;
// a head's bias slab is 16 rows of 72 halves plus 8: its stores from 8 heads at once fall in distinct banks
constexpr int kSlab = 16, kBiasRow = 72, kBiasHead = kSlab * kBiasRow + 8, kValueRow = 40;

FRY_DEVICE void mma_f16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// fp16 <-> fp32 off the conversion unit where possible: widening by the mixed-precision add, narrowing two at a time
FRY_DEVICE uint32_t pack_half2(float lo, float hi) { return pack_half2_rn(lo, hi); }
FRY_DEVICE float low_half(uint32_t pair) { return h2f_exact(static_cast<uint16_t>(pair & 0xffff)); }
FRY_DEVICE float high_half(uint32_t pair) { return h2f_exact(static_cast<uint16_t>(pair >> 16)); }
FRY_DEVICE float quad_sum(float v) {
    v += __shfl_xor_sync(0xffffffffu, v, 1);
    return v + __shfl_xor_sync(0xffffffffu, v, 2);
}
FRY_DEVICE float lane0(uint64_t v) { return lanes(v).x; }
FRY_DEVICE float lane1(uint64_t v) { return lanes(v).y; }
// the fp16 pair (low, high) as two fp32 lanes
FRY_DEVICE uint64_t widen2(uint32_t pair) { return pair2(low_half(pair), high_half(pair)); }
FRY_DEVICE uint32_t narrow2(uint64_t v) { return pack_half2(lane0(v), lane1(v)); }

FRY_DEVICE float quad_max(float v) {
    v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 1));
    return fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 2));
}

// paired[i][j][t] = templates[t][i][j]: a key's 8 templates side by side, the B operand of the bias MMA.
__global__ void pair_templates_kernel(const uint16_t* __restrict__ templates, uint16_t* __restrict__ paired) {
    grid_dependency_start();
    const int index = blockIdx.x * blockDim.x + threadIdx.x;  // over 64 x 64 (i, j)
    if (index >= kAttnSquares * kAttnSquares) return;
    uint16_t row[kAttnTemplates];
#pragma unroll
    for (int t = 0; t < kAttnTemplates; ++t) row[t] = templates[t * kAttnSquares * kAttnSquares + index];
    *reinterpret_cast<uint4*>(paired + index * kAttnTemplates) = *reinterpret_cast<const uint4*>(row);
}

// The template bias of square rows [16 * slab, 16 * slab + 16) for the CTA's heads into bias [head][kBiasHead] (fp16).
FRY_DEVICE void make_bias_slab(uint16_t* bias, const uint16_t* board, const uint16_t* paired, int slab, int width, int c_offset,
                               int first_head, int heads_here, int warp, int warps, int g, int t) {
    for (int pair = warp; pair < kSlab / 2; pair += warps) {
        const int i0 = slab * kSlab + 2 * pair, i1 = i0 + 1;
        uint32_t a0 = 0, a3 = 0;
        if (g < heads_here) {
            a0 = __ldcs(reinterpret_cast<const uint32_t*>(board + i0 * width + c_offset + (first_head + g) * kAttnTemplates + 2 * t));
            a3 = __ldcs(reinterpret_cast<const uint32_t*>(board + i1 * width + c_offset + (first_head + g) * kAttnTemplates + 2 * t));
        }
        const uint16_t* t0 = paired + (i0 * kAttnSquares + g) * kAttnTemplates + 2 * t;
        const uint16_t* t1 = paired + (i1 * kAttnSquares + g) * kAttnTemplates + 2 * t;
#pragma unroll
        for (int j = 0; j < kAttnSquares / 8; ++j) {
            float c[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            mma_f16(c, a0, 0u, 0u, a3, *reinterpret_cast<const uint32_t*>(t0 + j * 8 * kAttnTemplates),
                    *reinterpret_cast<const uint32_t*>(t1 + j * 8 * kAttnTemplates));
            if (g < heads_here) {
                uint16_t* to = bias + g * kBiasHead + 2 * pair * kBiasRow + j * 8 + 2 * t;
                *reinterpret_cast<uint32_t*>(to) = pack_half2(c[0], c[1]);
                *reinterpret_cast<uint32_t*>(to + kBiasRow) = pack_half2(c[2], c[3]);
            }
        }
    }
}

// Queries of rows [first, first + 16) for one head, raw (the A layout of m16n8k16: rows g and g + 8, depth 2t and 2t + 8).
template <int KS>
FRY_DEVICE void load_queries(uint32_t (&raw)[KS][2][2], const uint16_t* board, int first, int width, int head, int dq, int g, int t) {
#pragma unroll
    for (int ks = 0; ks < KS; ++ks)
#pragma unroll
        for (int r = 0; r < 2; ++r)
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                const int row = first + g + 8 * r, col = ks * 16 + half * 8 + 2 * t;
                raw[ks][r][half] = (row < kAttnTokens && col < dq) ? __ldcs(reinterpret_cast<const uint32_t*>(board + row * width + head * dq + col)) : 0u;
            }
}

// DQP: dq padded to the MMA depth (16 or 32). Shared: keys [kv][80][DQP + 8], values [kv][80][40], one bias slab (at most
// 70 KB). Two CTAs an SM, with up to 128 registers a thread: three (80 registers, some spilled) measured the same at 256
// boards and 3-6% slower at 8, 16 and 192.
// NORMED: the projected rows' query and key columns are already RMS-normalised with their gains (the projection GEMM's
// kEpiBiasQkNorm epilogue did it, to the same bits), so keys are copied and queries used as they are.
template <int DQP, bool NORMED>
__global__ void __launch_bounds__(kMaxHeadsPerCta * 32, 2)
    attention_kernel(const uint16_t* __restrict__ projected, const uint16_t* __restrict__ paired, const uint16_t* __restrict__ q_gain,
                     const uint16_t* __restrict__ k_gain, uint16_t* __restrict__ out, int heads, int kv_heads, int dq, float eps, float scale) {
    grid_dependency_start();
    constexpr int KROW = DQP + 8, KS = DQP / 16;
    extern __shared__ __align__(16) uint16_t attn_smem[];
    const int heads_here = blockDim.x / 32, warps = heads_here;
    const int group = heads / kv_heads;
    const int kv_here = heads_here / group;
    uint16_t* keys = attn_smem;                                   // [kv_here][80][KROW]
    uint16_t* values = keys + kv_here * kAttnKeys * KROW;         // [kv_here][80][kValueRow]
    uint16_t* bias = values + kv_here * kAttnKeys * kValueRow;    // [heads_here][16][kBiasRow]

    const int b = blockIdx.y, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
    const int width = (heads + kv_heads) * dq + kv_heads * kAttnDv + heads * kAttnTemplates;
    const int k_offset = heads * dq, v_offset = (heads + kv_heads) * dq, c_offset = v_offset + kv_heads * kAttnDv;
    const int first_head = blockIdx.x * heads_here, first_kv = blockIdx.x * kv_here;
    const uint16_t* board = projected + static_cast<size_t>(b) * kAttnTokens * width;
    // the mean of dq squares: for a power-of-two dq, the multiply by its reciprocal rounds exactly as the division
    const bool dq_pow2 = (dq & (dq - 1)) == 0;
    const float dq_reciprocal = 1.0f / static_cast<float>(dq);
    auto mean_of = [&](float sum) { return dq_pow2 ? __fmul_rn(sum, dq_reciprocal) : __fdiv_rn(sum, static_cast<float>(dq)); };

    // values as they are, [kv][key][dv], zero past the 70th key: 16-byte cp.async copies, a thread's all in flight at
    // once while the keys below are normalised; waited for before the first phase
    for (int item = tid; item < kv_here * kAttnKeys * (kAttnDv / 8); item += blockDim.x) {
        const int kv = item / (kAttnKeys * 4), rest = item % (kAttnKeys * 4), key = rest / 4, part = rest % 4;
        uint16_t* to = values + (kv * kAttnKeys + key) * kValueRow + part * 8;
        if (key < kAttnTokens) cp_async16(to, board + key * width + v_offset + (first_kv + kv) * kAttnDv + part * 8);
        else *reinterpret_cast<uint4*>(to) = make_uint4(0, 0, 0, 0);
    }
    cp_async_commit();
    // normalised keys (zero past dq and past the 70th key), 16-byte loads and stores; a thread's keys' loads are issued
    // together, ahead of their arithmetic
    constexpr int kKeyParts = DQP / 8;
    auto load_key = [&](int item, uint4 (&raw)[kKeyParts]) {
        const int kv = item / kAttnKeys, key = item % kAttnKeys;
        const uint16_t* from = board + key * width + k_offset + (first_kv + kv) * dq;
#pragma unroll
        for (int part = 0; part < kKeyParts; ++part)
            raw[part] = (key < kAttnTokens && part * 8 < dq) ? __ldcs(reinterpret_cast<const uint4*>(from + part * 8)) : make_uint4(0, 0, 0, 0);
    };
    auto store_key = [&](int item, const uint4 (&raw)[kKeyParts]) {
        const int kv = item / kAttnKeys, key = item % kAttnKeys;
        if constexpr (NORMED) {  // zero past dq and past the 70th key, as loaded
#pragma unroll
            for (int part = 0; part < kKeyParts; ++part) *reinterpret_cast<uint4*>(keys + (kv * kAttnKeys + key) * KROW + part * 8) = raw[part];
        } else {
            float k[DQP];
#pragma unroll
            for (int part = 0; part < kKeyParts; ++part) {
                const uint32_t words[4] = {raw[part].x, raw[part].y, raw[part].z, raw[part].w};
#pragma unroll
                for (int w = 0; w < 4; ++w) {
                    k[part * 8 + 2 * w] = low_half(words[w]);
                    k[part * 8 + 2 * w + 1] = high_half(words[w]);
                }
            }
            float squares = 0.0f;
#pragma unroll
            for (int i = 0; i < DQP; ++i) squares = __fmaf_rn(k[i], k[i], squares);
            const float inverse = rsqrtf(__fadd_rn(mean_of(squares), eps));
            uint16_t* row = keys + (kv * kAttnKeys + key) * KROW;
#pragma unroll
            for (int part = 0; part < kKeyParts; ++part) {
                uint32_t words[4];
#pragma unroll
                for (int w = 0; w < 4; ++w) {
                    const int i = part * 8 + 2 * w;
                    const float g0 = i < dq ? h2f_exact(k_gain[i]) : 0.0f, g1 = i + 1 < dq ? h2f_exact(k_gain[i + 1]) : 0.0f;
                    words[w] = key < kAttnTokens ? pack_half2(__fmul_rn(__fmul_rn(k[i], inverse), g0), __fmul_rn(__fmul_rn(k[i + 1], inverse), g1))
                                                 : 0u;
                }
                *reinterpret_cast<uint4*>(row + part * 8) = make_uint4(words[0], words[1], words[2], words[3]);
            }
        }
    };
    const int key_items = kv_here * kAttnKeys;
    for (int item = tid; item < key_items; item += 2 * blockDim.x) {
        const int second = item + blockDim.x;
        uint4 first_raw[kKeyParts], second_raw[kKeyParts];
        load_key(item, first_raw);
        if (second < key_items) load_key(second, second_raw);
        store_key(item, first_raw);
        if (second < key_items) store_key(second, second_raw);
    }
    // this CTA's phases: all five, or with a phase split (blockIdx.z, small batches), a share of them
    const int phases = (5 + gridDim.z - 1) / gridDim.z;
    const int phase_begin = blockIdx.z * phases, phase_end = min(5, phase_begin + phases);
    if (phase_begin >= 5) {  // uniform across the CTA; the launcher gives every group a phase
        cp_async_wait<0>();    // no copy may still be writing this CTA's shared memory when it leaves
        return;
    }
    if (phase_begin < 4) make_bias_slab(bias, board, paired, phase_begin, width, c_offset, first_head, heads_here, warp, warps, g, t);

    const int head = first_head + warp;
    const uint16_t* kv_keys = keys + (warp / group) * kAttnKeys * KROW;
    const uint16_t* kv_values = values + (warp / group) * kAttnKeys * kValueRow;
    float qg[KS][2][2] = {};  // the query gains (NORMED takes none: q_gain may be null)
    if constexpr (!NORMED) {
#pragma unroll
        for (int ks = 0; ks < KS; ++ks)
#pragma unroll
            for (int half = 0; half < 2; ++half)
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const int col = ks * 16 + half * 8 + 2 * t + e;
                    qg[ks][half][e] = col < dq ? h2f_exact(q_gain[col]) : 0.0f;
                }
    }
    uint32_t raw_q[KS][2][2];
    load_queries<KS>(raw_q, board, phase_begin * kSlab, width, head, dq, g, t);
    cp_async_wait<0>();  // this thread's value copies have landed; the barrier makes everyone's visible
    __syncthreads();

    const uint64_t scale2 = pair2(scale, scale), log2e2 = pair2(1.4426950408889634f, 1.4426950408889634f);
    // the metadata phase's rows g + 8 (72-79) do not exist: its r = 1 half is skipped
    constexpr int kRowHalves = 2;
    // one phase: 16 query rows from `first`; SQUARES (phases 0-3) adds the slab's template bias, the metadata phase (4)
    // has none and is the last
    auto run_phase = [&](auto squares_tag, int phase) {
        constexpr bool SQUARES = decltype(squares_tag)::value;
        const int first = phase * kSlab;
        // the next phase's queries, ahead of this phase's work
        uint32_t next_q[KS][2][2];
        if (SQUARES && phase + 1 < phase_end) load_queries<KS>(next_q, board, first + kSlab, width, head, dq, g, t);

        uint32_t a[KS][4];
#pragma unroll
        for (int r = 0; r < kRowHalves; ++r) {
            if (!SQUARES && r == 1) {
#pragma unroll
                for (int ks = 0; ks < KS; ++ks) a[ks][1] = a[ks][3] = 0u;
                continue;
            }
            if constexpr (NORMED) {
#pragma unroll
                for (int ks = 0; ks < KS; ++ks)
#pragma unroll
                    for (int half = 0; half < 2; ++half) a[ks][r + 2 * half] = raw_q[ks][r][half];
                continue;
            }
            float squares = 0.0f;
#pragma unroll
            for (int ks = 0; ks < KS; ++ks)
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    const float x0 = low_half(raw_q[ks][r][half]), x1 = high_half(raw_q[ks][r][half]);
                    squares = __fmaf_rn(x1, x1, __fmaf_rn(x0, x0, squares));
                }
            const float inverse = rsqrtf(__fadd_rn(mean_of(quad_sum(squares)), eps));
#pragma unroll
            for (int ks = 0; ks < KS; ++ks)
#pragma unroll
                for (int half = 0; half < 2; ++half)
                    a[ks][r + 2 * half] = pack_half2(__fmul_rn(__fmul_rn(low_half(raw_q[ks][r][half]), inverse), qg[ks][half][0]),
                                                     __fmul_rn(__fmul_rn(high_half(raw_q[ks][r][half]), inverse), qg[ks][half][1]));
        }
        // scores over the 9 key tiles that hold real keys (keys 72-79 never exist: their probabilities are 0), as fp32
        // pairs: s2[j][r] holds row g + 8 r, keys 8 j + 2 t and + 1
        constexpr int kTiles = 9;
        uint64_t s2[kTiles][2];
#pragma unroll
        for (int j = 0; j < kTiles; ++j) {
            float c[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            const uint16_t* key_row = kv_keys + (j * 8 + g) * KROW + 2 * t;
#pragma unroll
            for (int ks = 0; ks < KS; ++ks)
                mma_f16(c, a[ks][0], a[ks][1], a[ks][2], a[ks][3], *reinterpret_cast<const uint32_t*>(key_row + ks * 16),
                        *reinterpret_cast<const uint32_t*>(key_row + ks * 16 + 8));
            s2[j][0] = pair2(c[0], c[1]);
            s2[j][1] = pair2(c[2], c[3]);
        }
        // s * scale + bias (the bias on the square block only), keys 70 and 71 masked
        const uint16_t* head_bias = bias + warp * kBiasHead;
        const uint64_t masked = pair2(-INFINITY, -INFINITY);
        uint64_t top2[2] = {masked, masked};
#pragma unroll
        for (int j = 0; j < kTiles; ++j)
#pragma unroll
            for (int r = 0; r < kRowHalves; ++r) {
                if (!SQUARES && r == 1) {
                    s2[j][1] = 0;  // probability 0 for the rows that do not exist
                    continue;
                }
                uint64_t b2 = 0;  // +0.0 in both lanes
                if (SQUARES && j < 8) b2 = widen2(*reinterpret_cast<const uint32_t*>(head_bias + (g + 8 * r) * kBiasRow + j * 8 + 2 * t));
                uint64_t v = fma2(s2[j][r], scale2, b2);
                if (j == kTiles - 1 && t == 3) v = masked;  // keys 70, 71
                s2[j][r] = v;
                top2[r] = pair2(fmaxf(lane0(top2[r]), lane0(v)), fmaxf(lane1(top2[r]), lane1(v)));
            }
        // every warp has read this slab: the next one takes its place while the exponentials run
        if (SQUARES && phase + 1 < 4 && phase + 1 < phase_end) {
            __syncthreads();
            make_bias_slab(bias, board, paired, phase + 1, width, c_offset, first_head, heads_here, warp, warps, g, t);
        }
        uint64_t shift2[2];
        float top[2];
#pragma unroll
        for (int r = 0; r < kRowHalves; ++r) {
            if (!SQUARES && r == 1) continue;
            top[r] = quad_max(fmaxf(lane0(top2[r]), lane1(top2[r])));
            const float shift = -top[r] * 1.4426950408889634f;
            shift2[r] = pair2(shift, shift);
        }
        uint64_t total2[2] = {0, 0};
#pragma unroll
        for (int j = 0; j < kTiles; ++j)
#pragma unroll
            for (int r = 0; r < kRowHalves; ++r) {
                if (!SQUARES && r == 1) continue;
                const uint64_t x = fma2(s2[j][r], log2e2, shift2[r]);  // (s - top) log2 e
                const uint64_t p = pair2(ex2_approx_ftz(lane0(x)), ex2_approx_ftz(lane1(x)));
                s2[j][r] = p;
                total2[r] = add2(total2[r], p);
            }
        float inverse[2];
#pragma unroll
        for (int r = 0; r < kRowHalves; ++r) inverse[r] = (!SQUARES && r == 1) ? 0.0f : __frcp_rn(quad_sum(__fadd_rn(lane0(total2[r]), lane1(total2[r]))));
        float o[4][4];
#pragma unroll
        for (int n = 0; n < 4; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
#pragma unroll
        for (int kk = 0; kk < 5; ++kk) {
            const uint32_t p0 = narrow2(s2[2 * kk][0]), p1 = narrow2(s2[2 * kk][1]);
            const uint32_t p2 = 2 * kk + 1 < kTiles ? narrow2(s2[2 * kk + 1][0]) : 0u;
            const uint32_t p3 = 2 * kk + 1 < kTiles ? narrow2(s2[2 * kk + 1][1]) : 0u;
#pragma unroll
            for (int n = 0; n < 4; n += 2) {
                const uint16_t* rows = kv_values + (kk * 16 + ((lane >> 3) & 1) * 8 + (lane & 7)) * kValueRow + n * 8 + (lane >> 4) * 8;
                uint32_t b0, b1, b2, b3;
                asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                             : "=r"(b0), "=r"(b1), "=r"(b2), "=r"(b3)
                             : "r"(smem_addr(rows)));
                mma_f16(o[n], p0, p1, p2, p3, b0, b1);
                mma_f16(o[n + 1], p0, p1, p2, p3, b2, b3);
            }
        }
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const int row = first + g + 8 * r;
            if (row >= kAttnTokens) continue;
            uint16_t* to = out + (static_cast<size_t>(b) * kAttnTokens + row) * (heads * kAttnDv) + head * kAttnDv + 2 * t;
            const uint64_t inverse2 = pair2(inverse[r], inverse[r]);
#pragma unroll
            for (int n = 0; n < 4; ++n)
                *reinterpret_cast<uint32_t*>(to + n * 8) = narrow2(mul2(pair2(o[n][2 * r], o[n][2 * r + 1]), inverse2));
        }
        if (SQUARES) {
#pragma unroll
            for (int ks = 0; ks < KS; ++ks)
#pragma unroll
                for (int r = 0; r < 2; ++r)
#pragma unroll
                    for (int half = 0; half < 2; ++half) raw_q[ks][r][half] = next_q[ks][r][half];
            __syncthreads();
        }
    };
    for (int phase = phase_begin; phase < 4 && phase < phase_end; ++phase) run_phase(std::true_type{}, phase);
    if (phase_end == 5) run_phase(std::false_type{}, 4);
}

cudaError_t pair_templates(const uint16_t* templates, uint16_t* paired, cudaStream_t stream) {
    return launch_dependent(pair_templates_kernel, dim3((kAttnSquares * kAttnSquares + 255) / 256), dim3(256), 0, stream, templates, paired);
}

cudaError_t template_attention(const uint16_t* projected, const uint16_t* paired, const uint16_t* q_gain, const uint16_t* k_gain,
                               uint16_t* out, int B, int heads, int kv_heads, int dq, int dv, int templates_count, float eps,
                               cudaStream_t stream, std::string* error, bool qk_normed) {
    if (B <= 0) return cudaSuccess;
    const int group = kv_heads > 0 ? heads / kv_heads : 0;
    const int per_cta = heads < kMaxHeadsPerCta ? heads : kMaxHeadsPerCta;
    const int width = (heads + kv_heads) * dq + kv_heads * dv + heads * templates_count;
    if (dv != kAttnDv || templates_count != kAttnTemplates || dq < 1 || dq > 32 || dq % 8 || kv_heads <= 0 || heads % kv_heads ||
        heads % per_cta || per_cta % group || ((heads + kv_heads) * dq) % 8 || width % 8) {
        if (error)
            *error = "template attention takes dv 32, 8 templates, dq a multiple of 8 up to 32, and head groups that fit 8 heads a CTA; "
                     "got heads " + std::to_string(heads) + ", kv heads " + std::to_string(kv_heads) + ", dq " + std::to_string(dq) +
                     ", dv " + std::to_string(dv);
        return cudaErrorInvalidValue;
    }
    const int kv_per_cta = per_cta / group;
    const float scale = static_cast<float>(1.0 / std::sqrt(static_cast<double>(dq)));  // 1 / math.sqrt(dq), rounded once to fp32
    // small batches: the phases shared among up to 5 CTAs (each stages the keys and values again), as many as keep the
    // CTAs within 4.5 an SM, so more SMs share a board (measured: 3 an SM was 3-5% slower at 32 to 96 boards, 6 an SM
    // slower at 96 and 128)
    int device = 0, multiprocessors = 0;
    cudaError_t status = cudaGetDevice(&device);
    if (status == cudaSuccess) status = cudaDeviceGetAttribute(&multiprocessors, cudaDevAttrMultiProcessorCount, device);
    if (status != cudaSuccess) return status;
    // 1, 2, 3 or 5 groups: each has a phase (4 groups of 2 phases would leave the last without one). Three groups only
    // from 4 fit: at 64 boards (3.5 fit) two groups measured 17.8 / 22.0 us a launch (dq 16 / 24) against 18.2 / 23.4
    const int ctas = heads / per_cta * B, fit = 9 * multiprocessors / (2 * ctas);
    const dim3 grid(heads / per_cta, B, fit >= 5 ? 5 : fit >= 4 ? 3 : fit >= 2 ? 2 : 1);
    const int dqp = dq <= 16 ? 16 : 32;
    const size_t bytes = (static_cast<size_t>(kv_per_cta) * kAttnKeys * (dqp + 8) + static_cast<size_t>(kv_per_cta) * kAttnKeys * kValueRow +
                          static_cast<size_t>(per_cta) * kBiasHead) * sizeof(uint16_t);
    if (qk_normed && dq != 8 && dq != 16 && dq != 24) {
        if (error) *error = "template attention takes normalised queries and keys for dq 8, 16 or 24 only";
        return cudaErrorInvalidValue;
    }
    auto run = [&](auto kernel) {
        const cudaError_t attribute = ensure_smem(reinterpret_cast<const void*>(kernel), static_cast<int>(bytes));
        if (attribute != cudaSuccess) return attribute;
        return launch_dependent(kernel, grid, dim3(per_cta * 32), bytes, stream, projected, paired, q_gain, k_gain, out, heads, kv_heads, dq, eps,
                                scale);
    };
    if (qk_normed) return dqp == 16 ? run(attention_kernel<16, true>) : run(attention_kernel<32, true>);
    return dqp == 16 ? run(attention_kernel<16, false>) : run(attention_kernel<32, false>);
}

}  // namespace fry
