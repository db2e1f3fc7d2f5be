// The heads after the last block: stream [B, 70, d] fp16 -> answer rows [B, 1969] fp32 (1968 move logits, then the
// expected score). The reference's B200 path is the torch one of `FusedTransformer.forward` (model/fused_blocks.py:863-874)
// with the weights folded by `head_weights` (:815-824), and `answer_rows` (engine/inference.py:19-23):
//
//   y = RMSNorm(x) in fp16;  a = y . A + a_bias (A = W_f^T W_t / sqrt d in fp16, fp32 accumulate);
//   narrow = y . N^T + n_bias (fp32): s (1), the 4 promotion logits, the 16 board-down units;
//   logit[f, t] = a_f . y_t + s_f, gathered to the 1968 moves, promotions plus their piece's logit at the landing square;
//   value = Linear(GELU(Linear(GELU(board-down) flattened))) ; score = softmax(value) . bin centres.
//
// Kernels: rms_norm (rows.cu); the tcgen05 f16 GEMM for a (gemm.cu); narrow_kernel (split-fp16 mma.sync, N = hi + lo /
// 2048, and the eval head's GELU'd inputs); policy_kernel (per board, the 64x64 logits by split-fp16 mma.sync, a = hi +
// lo / 2048, so the products stay fp32-exact); the eval head's two layers as split-K partial products
// (linear_split_kernel) summed in a fixed order by linear_sum_kernel; expected_score_kernel (softmax times the bin
// centres). fp32 arithmetic throughout, where the reference uses tf32 matmuls.
#include <string>

#include "common.cuh"
#include "kernels.h"
#include "moves.h"

namespace fry {

constexpr int kHeadTokens = 70, kHeadSquares = 64, kNarrow = 21, kNarrowStride = 24, kDown = 16, kMoves = 1968;
constexpr int kEvalInputs = kHeadTokens * kDown;  // the eval head's first layer takes 70 x 16 GELU'd board-down units
constexpr float kLoScale = 2048.0f;
constexpr int kLinearTile = 64, kLinearStep = 16;  // linear_split_kernel: 64 boards x 64 outputs a CTA, K in steps of 16
static_assert(kLinearTile * kLinearStep == 4 * 256, "linear_split_kernel: one float4 of x and of W a thread a step");
constexpr int kEvalSplits = 8;  // the eval head's layers: K in 8 splits, whatever the batch
// narrow_kernel: the 21 outputs padded to 3 mma tiles of 8; 8 tiles of 16 rows a CTA, the columns in kNarrowParts parts
constexpr int kNarrowTile = 24, kNarrowTiles = 8, kNarrowParts = 2, kNarrowLoads = 12;
constexpr int kNarrowAhead = 4;  // narrow_kernel: steps of 16 columns loading ahead of the MMAs
// policy_kernel: chunks of 64 columns in a ring of 3 stages; row pitches padded by 8 elements (conflict-free fragment loads)
constexpr int kPolicyChunk = 64, kPolicyStages = 3, kPolicyAPitch = kPolicyChunk + 8, kPolicyYPitch = kPolicyChunk + 8;
static_assert(kHeadSquares * (kHeadSquares + 1) <= kPolicyStages * kHeadSquares * kPolicyAPitch, "the logits fit in the a chunks");

FRY_DEVICE float gelu(float x) { return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f)); }

size_t heads_workspace_bytes(int B, int D) { return heads_workspace_bytes_of(B, D); }

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

// narrow[m, 0..20] = y[m] . N^T + n_bias on the tensor cores: N (fp32) split into fp16 halves N = hi + lo / 2048 in shared
// memory, [24][D + 8] each (rows 21..23 zero; the 8-element pad puts a fragment's 32 lanes on 32 banks), and y times both
// halves by split-fp16 mma.sync (y is fp16, so every product is fp32-exact, as in policy_kernel). A CTA takes 8 tiles of
// 16 rows; warp w works on tile w % 8 over the (w / 8)-th of kNarrowParts parts of the columns, and the parts' sums are
// added in order through shared memory. eval_in[b, t * 16 + i] = GELU(narrow[b * 70 + t, 5 + i]), the eval head's
// inputs, once per board. The weights are the network's constants and are split before the wait on the kernel ahead.
__global__ void __launch_bounds__(kNarrowTiles * kNarrowParts * 32) narrow_kernel(const uint16_t* __restrict__ y,
                                                                                  const float* __restrict__ weight,
                                                                                  const float* __restrict__ bias, float* __restrict__ narrow,
                                                                                  float* __restrict__ eval_in, int M, int D) {
    extern __shared__ __align__(16) uint16_t narrow_split[];
    const int pitch = D + 8, quads = kNarrowTile * D / 4, per_row = D / 4;
    uint16_t* w_hi = narrow_split;
    uint16_t* w_lo = narrow_split + kNarrowTile * pitch;
    float* part_sums = reinterpret_cast<float*>(narrow_split + 2 * kNarrowTile * pitch);  // [parts - 1][tiles][32][13]
    for (int base = threadIdx.x; base < quads; base += blockDim.x * kNarrowLoads) {
        float4 v[kNarrowLoads];
#pragma unroll
        for (int u = 0; u < kNarrowLoads; ++u) {
            const int i = base + u * blockDim.x, j = i / per_row;
            v[u] = (i < quads && j < kNarrow) ? __ldg(reinterpret_cast<const float4*>(weight + static_cast<size_t>(i) * 4))
                                              : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
#pragma unroll
        for (int u = 0; u < kNarrowLoads; ++u) {
            const int i = base + u * blockDim.x, j = i / per_row, k = (i % per_row) * 4;
            if (i < quads) {
                uint32_t hi01, lo01, hi23, lo23;
                split_pair(make_float2(v[u].x, v[u].y), hi01, lo01);
                split_pair(make_float2(v[u].z, v[u].w), hi23, lo23);
                *reinterpret_cast<uint2*>(w_hi + j * pitch + k) = make_uint2(hi01, hi23);
                *reinterpret_cast<uint2*>(w_lo + j * pitch + k) = make_uint2(lo01, lo23);
            }
        }
    }
    grid_dependency_start();
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int tile = warp % kNarrowTiles, part = warp / kNarrowTiles, first = (blockIdx.x * kNarrowTiles + tile) * 16;
    const int steps = D / 16, k_begin = steps * part / kNarrowParts * 16, k_end = steps * (part + 1) / kNarrowParts * 16;
    // rows past M compute on row M - 1 and are not written
    const uint16_t* rows[2] = {y + static_cast<size_t>(min(first + g, M - 1)) * D + 2 * t,
                               y + static_cast<size_t>(min(first + g + 8, M - 1)) * D + 2 * t};
    float hi[3][4], lo[3][4];
#pragma unroll
    for (int n = 0; n < 3; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) hi[n][e] = lo[n][e] = 0.0f;
    uint32_t a_next[kNarrowAhead][4];
    auto fetch = [&](int slot, int k) {
        a_next[slot][0] = *reinterpret_cast<const uint32_t*>(rows[0] + k);
        a_next[slot][1] = *reinterpret_cast<const uint32_t*>(rows[1] + k);
        a_next[slot][2] = *reinterpret_cast<const uint32_t*>(rows[0] + k + 8);
        a_next[slot][3] = *reinterpret_cast<const uint32_t*>(rows[1] + k + 8);
    };
    const bool active = first < M;
    if (active) {
#pragma unroll
        for (int slot = 0; slot < kNarrowAhead; ++slot)
            if (k_begin + slot * 16 < k_end) fetch(slot, k_begin + slot * 16);
        const uint16_t* b_hi = w_hi + g * pitch + 2 * t;
        const uint16_t* b_lo = w_lo + g * pitch + 2 * t;
        for (int k0 = k_begin; k0 < k_end; k0 += 16 * kNarrowAhead) {
#pragma unroll
            for (int slot = 0; slot < kNarrowAhead; ++slot) {
                const int k = k0 + slot * 16;
                if (k < k_end) {
                    const uint32_t a[4] = {a_next[slot][0], a_next[slot][1], a_next[slot][2], a_next[slot][3]};
                    if (k + 16 * kNarrowAhead < k_end) fetch(slot, k + 16 * kNarrowAhead);
#pragma unroll
                    for (int n = 0; n < 3; ++n) {
                        const uint16_t* h = b_hi + n * 8 * pitch + k;
                        const uint16_t* l = b_lo + n * 8 * pitch + k;
                        mma_f16_heads(hi[n], a, *reinterpret_cast<const uint32_t*>(h), *reinterpret_cast<const uint32_t*>(h + 8));
                        mma_f16_heads(lo[n], a, *reinterpret_cast<const uint32_t*>(l), *reinterpret_cast<const uint32_t*>(l + 8));
                    }
                }
            }
        }
    }
    float sums[3][4];
#pragma unroll
    for (int n = 0; n < 3; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) sums[n][e] = __fadd_rn(hi[n][e], __fdiv_rn(lo[n][e], kLoScale));
    if (kNarrowParts > 1) {
        if (part > 0) {
            float* mine = part_sums + ((part - 1) * kNarrowTiles + tile) * 32 * 13 + lane * 13;
#pragma unroll
            for (int i = 0; i < 12; ++i) mine[i] = sums[i >> 2][i & 3];
        }
        __syncthreads();
        if (part > 0) return;
#pragma unroll
        for (int p = 1; p < kNarrowParts; ++p) {
            const float* theirs = part_sums + ((p - 1) * kNarrowTiles + tile) * 32 * 13 + lane * 13;
#pragma unroll
            for (int i = 0; i < 12; ++i) sums[i >> 2][i & 3] = __fadd_rn(sums[i >> 2][i & 3], theirs[i]);
        }
    }
    if (!active) return;
#pragma unroll
    for (int n = 0; n < 3; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int m = first + g + (e >> 1) * 8, j = n * 8 + 2 * t + (e & 1);
            if (m < M && j < kNarrow) {
                const float value = __fadd_rn(sums[n][e], bias[j]);
                narrow[static_cast<size_t>(m) * kNarrowStride + j] = value;
                if (j >= 5) eval_in[static_cast<size_t>(m / kHeadTokens) * kEvalInputs + (m % kHeadTokens) * kDown + j - 5] = gelu(value);
            }
        }
}


// One CTA (8 warps) per (board, Q-th of the from-squares): its 64 / Q rows of L = a_sq . y_sq^T (64 x 64), then the
// move logits of the moves from those squares. The CTA's square rows of a (fp32) and the board's 64 of y (fp16) stream
// through shared memory in chunks of kPolicyChunk columns, kPolicyStages deep, by 16-byte cp.async (whole 128-byte lines
// per 8 lanes); each warp takes its 16 x 32 / Q tile of L from fragments read out of shared memory, the padded pitches
// putting each fragment load on distinct banks. Q = 1 but at a few boards, which split a board over 4 CTAs. Each
// logit's sums run in the same order whatever Q, so the rows do not depend on it.
template <int Q>
__global__ void __launch_bounds__(256) policy_kernel(const float* __restrict__ a, const uint16_t* __restrict__ y,
                                                     const float* __restrict__ narrow, float* __restrict__ rows, int D) {
    static_assert(Q == 1 || Q == 2 || Q == 4, "a board's from-squares in 1, 2 or 4 parts");
    constexpr int kRowsHere = kHeadSquares / Q, kNt = 4 / Q;  // a's rows this CTA; n tiles of 8 a warp
    extern __shared__ __align__(16) float policy_smem[];  // a chunks, then y chunks; the logits reuse the a chunks at the end
    auto a_chunks = reinterpret_cast<float(*)[kHeadSquares * kPolicyAPitch]>(policy_smem);
    auto y_chunks = reinterpret_cast<uint16_t(*)[kHeadSquares * kPolicyYPitch]>(policy_smem + kPolicyStages * kHeadSquares * kPolicyAPitch);
    auto logits = reinterpret_cast<float(*)[kHeadSquares + 1]>(policy_smem);
    grid_dependency_start();
    const int b = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    // this CTA's from-squares [row0, row0 + kRowsHere); 2 Q warps a 16-row m tile, each with kNt n tiles
    const int row0 = blockIdx.y * kRowsHere, m_tile = warp / (2 * Q), n_first = (warp % (2 * Q)) * kNt;
    const size_t board = static_cast<size_t>(b) * kHeadTokens;
    const int chunks = (D + kPolicyChunk - 1) / kPolicyChunk;
    auto load_chunk = [&](int chunk) {
        const int stage = chunk % kPolicyStages, k0 = chunk * kPolicyChunk;
        constexpr int a_pieces = kPolicyChunk / 4, y_pieces = kPolicyChunk / 8;  // 16-byte pieces of a row
#pragma unroll
        for (int i = threadIdx.x; i < kRowsHere * a_pieces; i += 256) {
            const int r = i / a_pieces, piece = i % a_pieces, k = k0 + piece * 4;
            if (k < D) cp_async16(&a_chunks[stage][r * kPolicyAPitch + piece * 4], a + (board + row0 + r) * D + k);
        }
#pragma unroll
        for (int i = threadIdx.x; i < kHeadSquares * y_pieces; i += 256) {
            const int r = i / y_pieces, piece = i % y_pieces, k = k0 + piece * 8;
            if (k < D) cp_async16(&y_chunks[stage][r * kPolicyYPitch + piece * 8], y + (board + r) * D + k);
        }
    };
#pragma unroll
    for (int chunk = 0; chunk < kPolicyStages - 1; ++chunk) {
        if (chunk < chunks) load_chunk(chunk);
        cp_async_commit();
    }
    float hi[kNt][4], lo[kNt][4];
#pragma unroll
    for (int n = 0; n < kNt; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) hi[n][e] = lo[n][e] = 0.0f;
    for (int chunk = 0; chunk < chunks; ++chunk) {
        cp_async_wait<kPolicyStages - 2>();
        __syncthreads();  // the chunk is in; and every warp is done with the stage the next load overwrites
        if (chunk + kPolicyStages - 1 < chunks) load_chunk(chunk + kPolicyStages - 1);
        cp_async_commit();
        const float* as = a_chunks[chunk % kPolicyStages] + (m_tile * 16 + g) * kPolicyAPitch + 2 * t;
        const uint16_t* ys = y_chunks[chunk % kPolicyStages] + (n_first * 8 + g) * kPolicyYPitch + 2 * t;
#pragma unroll
        for (int kk = 0; kk < kPolicyChunk; kk += 16) {
            if (chunk * kPolicyChunk + kk < D) {
                const float2 a_pairs[4] = {*reinterpret_cast<const float2*>(as + kk), *reinterpret_cast<const float2*>(as + 8 * kPolicyAPitch + kk),
                                           *reinterpret_cast<const float2*>(as + kk + 8),
                                           *reinterpret_cast<const float2*>(as + 8 * kPolicyAPitch + kk + 8)};
                uint32_t ah[4], al[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) split_pair(a_pairs[i], ah[i], al[i]);
#pragma unroll
                for (int n = 0; n < kNt; ++n) {
                    const uint16_t* yn = ys + n * 8 * kPolicyYPitch + kk;
                    const uint32_t b0 = *reinterpret_cast<const uint32_t*>(yn), b1 = *reinterpret_cast<const uint32_t*>(yn + 8);
                    mma_f16_heads(hi[n], ah, b0, b1);
                    mma_f16_heads(lo[n], al, b0, b1);
                }
            }
        }
    }
    cp_async_wait<0>();
    __syncthreads();  // every warp is done reading the chunks the logits overwrite
#pragma unroll
    for (int n = 0; n < kNt; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int row = m_tile * 16 + g + (e >> 1) * 8, col = (n_first + n) * 8 + 2 * t + (e & 1);
            logits[row][col] = __fadd_rn(hi[n][e], __fdiv_rn(lo[n][e], kLoScale));
        }
    __syncthreads();
    const float* board_narrow = narrow + board * kNarrowStride;
    for (int m = threadIdx.x; m < kMoves; m += blockDim.x) {
        const int pair = kMovePairs[m], from = pair >> 6, to = pair & 63;
        if (from < row0 || from >= row0 + kRowsHere) continue;  // another CTA's square
        float logit = __fadd_rn(logits[from - row0][to], board_narrow[from * kNarrowStride]);
        const int promotion = kMovePromotion[m];
        if (promotion >= 0) logit = __fadd_rn(logit, board_narrow[to * kNarrowStride + 1 + promotion]);
        rows[static_cast<size_t>(b) * (kMoves + 1) + m] = logit;
    }
}

// One split of an fp32 linear layer: partial[split, b, u] = sum over inputs i of split's K range of W[u, i] * x[b, i], for
// x [B, K] and W [N, K] row-major (K a multiple of 4, both 16-byte aligned). A CTA takes 64 boards x 64 outputs of one
// split, 4 x 4 a thread, K in steps of 16 through shared memory (transposed, two buffers): each thread loads one float4
// of x and of W a step, the next step's while this one's FMAs run. Each output's sum runs over its split's inputs in
// order, whatever the batch.
__global__ void __launch_bounds__(256) linear_split_kernel(const float* __restrict__ x, const float* __restrict__ weight,
                                                           float* __restrict__ partial, int B, int K, int N, int k_split) {
    grid_dependency_start();
    __shared__ __align__(16) float xs[2][kLinearStep][kLinearTile + 4];
    __shared__ __align__(16) float ws[2][kLinearStep][kLinearTile + 4];
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int b0 = blockIdx.y * kLinearTile, u0 = blockIdx.x * kLinearTile;
    const int k_begin = blockIdx.z * k_split, k_end = min(K, k_begin + k_split);
    const int load_row = threadIdx.x >> 2, load_quad = threadIdx.x & 3, board = b0 + load_row, unit = u0 + load_row;
    const float* x_row = x + static_cast<size_t>(min(board, B - 1)) * K + load_quad * 4;
    const float* w_row = weight + static_cast<size_t>(min(unit, N - 1)) * K + load_quad * 4;
    const float4 zero = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    float4 xv, wv;
    auto fetch = [&](int k0) {
        const bool in = k0 + load_quad * 4 < k_end;
        xv = in && board < B ? *reinterpret_cast<const float4*>(x_row + k0) : zero;
        wv = in && unit < N ? __ldg(reinterpret_cast<const float4*>(w_row + k0)) : zero;
    };
    auto stash = [&](int buffer) {
        float* xc = &xs[buffer][load_quad * 4][load_row];
        float* wc = &ws[buffer][load_quad * 4][load_row];
        xc[0] = xv.x, xc[kLinearTile + 4] = xv.y, xc[2 * (kLinearTile + 4)] = xv.z, xc[3 * (kLinearTile + 4)] = xv.w;
        wc[0] = wv.x, wc[kLinearTile + 4] = wv.y, wc[2 * (kLinearTile + 4)] = wv.z, wc[3 * (kLinearTile + 4)] = wv.w;
    };
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;
    fetch(k_begin);
    stash(0);
    __syncthreads();
    int buffer = 0;
    for (int k0 = k_begin; k0 < k_end; k0 += kLinearStep) {
        const bool more = k0 + kLinearStep < k_end;
        if (more) fetch(k0 + kLinearStep);
#pragma unroll
        for (int kk = 0; kk < kLinearStep; ++kk) {
            const float4 a = *reinterpret_cast<const float4*>(&xs[buffer][kk][ty * 4]);
            const float4 w = *reinterpret_cast<const float4*>(&ws[buffer][kk][tx * 4]);
            const float av[4] = {a.x, a.y, a.z, a.w}, wv4[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = __fmaf_rn(av[i], wv4[j], acc[i][j]);
        }
        if (more) stash(buffer ^ 1);
        __syncthreads();
        buffer ^= 1;
    }
    float* out = partial + static_cast<size_t>(blockIdx.z) * B * N;
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int b = b0 + ty * 4 + i, u = u0 + tx * 4 + j;
            if (b < B && u < N) out[static_cast<size_t>(b) * N + u] = acc[i][j];
        }
}

// out[b, u] = act(bias[u] + sum over splits s = 0, 1, ... of partial[s, b, u]), GELU when GELU.
template <bool GELU>
__global__ void __launch_bounds__(256) linear_sum_kernel(const float* __restrict__ partial, const float* __restrict__ bias,
                                                         float* __restrict__ out, int B, int N, int splits) {
    grid_dependency_start();
    const int index = blockIdx.x * blockDim.x + threadIdx.x;
    if (index >= B * N) return;
    float total = partial[index];
    for (int split = 1; split < splits; ++split) total = __fadd_rn(total, partial[static_cast<size_t>(split) * B * N + index]);
    const float value = __fadd_rn(total, bias[index % N]);
    out[index] = GELU ? gelu(value) : value;
}

// Splits of K for the eval head's layers: kEvalSplits of whole steps of 16 (a board's sums do not depend on its batch).
inline int split_size(int K) { return ((K + kEvalSplits - 1) / kEvalSplits + kLinearStep - 1) / kLinearStep * kLinearStep; }
static_assert(kEvalSplits <= kEvalSplitsMax, "the workspace holds kEvalSplitsMax splits");

// One warp per board: the softmax of its value logits times the bin centres (2i + 1) / 2bins, into the row's last column.
// With lean lanes, each board's answer also gathers its lane's answer columns of its row (the move logits the policy
// kernel wrote, the expected score this one writes): lean_answers[b, k] = rows[b, column k], a column outside the row
// recorded as kBadColumn and answered 0.
__global__ void __launch_bounds__(256) expected_score_kernel(const float* __restrict__ logits, float* __restrict__ rows, int B, int bins,
                                                             const uint8_t* __restrict__ lean_rows, float* __restrict__ lean_answers) {
    grid_dependency_start();
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
    const float expected = __fdiv_rn(weighted, total);
    float* row_out = rows + static_cast<size_t>(b) * (kMoves + 1);
    if (lane == 0) row_out[kMoves] = expected;
    if (lean_answers) {
        __syncwarp();  // the expected score, which padding columns gather, is in the row
        const uint8_t* columns = lean_rows + static_cast<size_t>(b) * kLeanRow + kHeadTokens;
        for (int k = lane; k < kLeanColumns; k += 32) {
            const int column = static_cast<int16_t>(static_cast<uint16_t>(columns[2 * k] | (columns[2 * k + 1] << 8)));
            const bool ok = column >= 0 && column <= kMoves;
            if (!ok) record_error(kBadColumn, b);
            lean_answers[static_cast<size_t>(b) * kLeanColumns + k] = ok ? (column == kMoves ? expected : row_out[column]) : 0.0f;
        }
    }
}

cudaError_t heads(const uint16_t* stream_x, const HeadWeights& w, float eps, float* rows, void* workspace, size_t workspace_bytes, int B,
                  int D, cudaStream_t stream, std::string* error, const uint8_t* lean_rows, float* lean_answers) {
    if (B <= 0) return cudaSuccess;
    if (D < 16 || D % 16 != 0 || D > 1024 || w.bins < 2 || w.bins > 256) {
        if (error) *error = "the heads take d_model a multiple of 16 from 16 to 1024 and 2 to 256 value bins";
        return cudaErrorInvalidValue;
    }
    if (workspace_bytes < heads_workspace_bytes(B, D)) {
        if (error) *error = "the heads' workspace is smaller than fry_heads_workspace_bytes";
        return cudaErrorInvalidValue;
    }
    if (reinterpret_cast<uintptr_t>(w.narrow_weight) % 16 != 0 || reinterpret_cast<uintptr_t>(w.hidden_weight) % 16 != 0 ||
        reinterpret_cast<uintptr_t>(w.out_weight) % 16 != 0) {
        if (error) *error = "the heads take the narrow and eval-head weights 16-byte aligned";
        return cudaErrorInvalidValue;
    }
    const int M = B * kHeadTokens;
    const HeadsWorkspace layout(B, D);
    uint8_t* base = static_cast<uint8_t*>(workspace);
    uint16_t* y = reinterpret_cast<uint16_t*>(base + layout.y);
    float* a = reinterpret_cast<float*>(base + layout.a);
    float* narrow = reinterpret_cast<float*>(base + layout.narrow);
    float* eval_in = reinterpret_cast<float*>(base + layout.eval_in);
    float* partial = reinterpret_cast<float*>(base + layout.partial);
    float* hidden = reinterpret_cast<float*>(base + layout.hidden);
    float* value_logits = reinterpret_cast<float*>(base + layout.logits);

    cudaError_t status = rms_norm_f16(stream_x, w.ln_gain, eps, y, M, D, stream);
    if (status != cudaSuccess) return status;
    GemmArgs args;
    args.bias_f32 = w.a_bias;
    args.out = a;
    status = gemm(1, kEpiLinearF32, y, w.a_weight, args, M, D, D, stream, error);
    if (status != cudaSuccess) return status;
    const size_t narrow_smem = 2ull * kNarrowTile * (D + 8) * sizeof(uint16_t) + (kNarrowParts - 1) * kNarrowTiles * 32 * 13 * sizeof(float);
    status = ensure_smem(reinterpret_cast<const void*>(narrow_kernel), static_cast<int>(narrow_smem));
    if (status != cudaSuccess) return status;
    status = launch_dependent(narrow_kernel, dim3((M + kNarrowTiles * 16 - 1) / (kNarrowTiles * 16)), dim3(kNarrowTiles * kNarrowParts * 32),
                              narrow_smem, stream, y, w.narrow_weight, w.narrow_bias, narrow, eval_in, M, D);
    if (status != cudaSuccess) return status;
    const size_t policy_smem = kPolicyStages * kHeadSquares * (kPolicyAPitch * sizeof(float) + kPolicyYPitch * sizeof(uint16_t));
    // a board's from-squares over 4 CTAs while that leaves at least half the SMs idle: at 1 board the forward 918 -> 912
    // us; at 64 and 256 boards, the 4 CTAs a board measured slower (1.822 -> 1.830, 4.75 -> 4.78 ms)
    int device = 0, multiprocessors = 0;
    status = cudaGetDevice(&device);
    if (status == cudaSuccess) status = cudaDeviceGetAttribute(&multiprocessors, cudaDevAttrMultiProcessorCount, device);
    if (status != cudaSuccess) return status;
    auto run_policy = [&](auto kernel, int parts) {
        cudaError_t attribute = ensure_smem(reinterpret_cast<const void*>(kernel), static_cast<int>(policy_smem));
        if (attribute != cudaSuccess) return attribute;
        return launch_dependent(kernel, dim3(B, parts), dim3(256), policy_smem, stream, a, y, narrow, rows, D);
    };
    status = 8 * B <= multiprocessors ? run_policy(policy_kernel<4>, 4) : run_policy(policy_kernel<1>, 1);
    if (status != cudaSuccess) return status;
    // the eval head: hidden = GELU(W1 . eval_in + b1), logits = W2 . hidden + b2, each as split-K partial products
    const int split1 = split_size(kEvalInputs), splits1 = (kEvalInputs + split1 - 1) / split1;
    status = launch_dependent(linear_split_kernel, dim3((D + kLinearTile - 1) / kLinearTile, (B + kLinearTile - 1) / kLinearTile, splits1),
                              dim3(256), 0, stream, eval_in, w.hidden_weight, partial, B, kEvalInputs, D, split1);
    if (status != cudaSuccess) return status;
    status = launch_dependent(linear_sum_kernel<true>, dim3((B * D + 255) / 256), dim3(256), 0, stream, partial, w.hidden_bias, hidden, B, D,
                              splits1);
    if (status != cudaSuccess) return status;
    const int split2 = split_size(D), splits2 = (D + split2 - 1) / split2;
    status = launch_dependent(linear_split_kernel, dim3((w.bins + kLinearTile - 1) / kLinearTile, (B + kLinearTile - 1) / kLinearTile, splits2),
                              dim3(256), 0, stream, hidden, w.out_weight, partial, B, D, w.bins, split2);
    if (status != cudaSuccess) return status;
    status = launch_dependent(linear_sum_kernel<false>, dim3((B * w.bins + 255) / 256), dim3(256), 0, stream, partial, w.out_bias, value_logits,
                              B, w.bins, splits2);
    if (status != cudaSuccess) return status;
    return launch_dependent(expected_score_kernel, dim3((B + 7) / 8), dim3(256), 0, stream, value_logits, rows, B, w.bins, lean_rows,
                            lean_answers);
}

}  // namespace fry
