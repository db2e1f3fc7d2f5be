// Row kernels of the Fry forward: HBM/L2-bound, one warp per activation row, 16-byte vector loads.
//
//  norm_quant_kernel    `norm_quant` / `mix_norm_quant` (model/int8_blocks.py:156-212): optional input mix, RMSNorm with
//                       gain in fp32, per-row absmax, int8 by round-half-even, scale absmax / 127.
//  rms_norm_kernel      the final nn.RMSNorm in fp16 (model/fused_blocks.py:863) ahead of the heads.
//  rotate_quant_kernel  `rotate_quant` (model/int8_blocks.py:216-251): the SwiGLU output zero-padded to the down width,
//                       times the block-diagonal 32x32 Sylvester Hadamard matrix (butterflies in registers and across
//                       each quad of lanes), per-row absmax, int8.
//  embedding_kernel     `board_embedding` (model/fused_blocks.py:449-507): embed[token] + position[t] + the 23 square
//                       feature rows of `SquareFeatures.indices` (model/model.py:147-169), found in-kernel from the board.
#include "common.cuh"
#include "kernels.h"

namespace fry {

constexpr int kRowWarps = 8;

FRY_DEVICE void unpack8(const uint4& u, float (&v)[8]) {
    const uint16_t* h = reinterpret_cast<const uint16_t*>(&u);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = h2f_bits(h[i]);
}

// x [M, D] fp16 -> q [M, D] int8, scale [M]; with MIX, x is first mixed with original and the mix stored to mixed.
// A warp takes ROWS consecutive rows and issues all their loads (and the gain's) before working on any, so the row
// latencies overlap; each row's arithmetic is the single-row order: per lane over its chunks, then the warp's tree.
template <int CHUNKS, bool MIX, int ROWS>
__global__ void __launch_bounds__(kRowWarps * 32) norm_quant_kernel(const uint16_t* __restrict__ x, const uint16_t* __restrict__ original,
                                                                    const uint16_t* residual_scale, const uint16_t* input_scale,
                                                                    const uint16_t* __restrict__ gain, float eps, uint16_t* mixed,
                                                                    int8_t* __restrict__ q, float* __restrict__ scale, int M, int D) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int first_row = (blockIdx.x * kRowWarps + warp) * ROWS;
    if (first_row >= M) return;
    float rs = 0.0f, is = 0.0f;
    if constexpr (MIX) {
        rs = h2f_bits(*residual_scale);
        is = h2f_bits(*input_scale);
    }
    uint4 raw[ROWS][CHUNKS], raw_original[MIX ? ROWS : 1][CHUNKS], raw_gain[CHUNKS];
#pragma unroll
    for (int c = 0; c < CHUNKS; ++c) {
        const int col = (c * 32 + lane) * 8;
        raw_gain[c] = col < D ? *reinterpret_cast<const uint4*>(gain + col) : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int r = 0; r < ROWS; ++r) {
            const bool ok = col < D && first_row + r < M;
            const size_t at = static_cast<size_t>(first_row + r) * D + col;
            raw[r][c] = ok ? *reinterpret_cast<const uint4*>(x + at) : make_uint4(0, 0, 0, 0);
            if constexpr (MIX) raw_original[r][c] = ok ? *reinterpret_cast<const uint4*>(original + at) : make_uint4(0, 0, 0, 0);
        }
    }
#pragma unroll
    for (int r = 0; r < ROWS; ++r) {
        const int row = first_row + r;
        if (row >= M) break;  // uniform across the warp
        const size_t base = static_cast<size_t>(row) * D;
        float v[CHUNKS][8];
        float squares = 0.0f;
#pragma unroll
        for (int c = 0; c < CHUNKS; ++c) {
            const int col = (c * 32 + lane) * 8;
            unpack8(raw[r][c], v[c]);
            if (col < D) {
                if constexpr (MIX) {
                    float o[8];
                    unpack8(raw_original[r][c], o);
                    uint16_t packed[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        packed[i] = f2h_bits(__fmaf_rn(rs, v[c][i], __fmul_rn(is, o[i])));
                        v[c][i] = h2f_bits(packed[i]);
                    }
                    *reinterpret_cast<uint4*>(mixed + base + col) = *reinterpret_cast<const uint4*>(packed);
                }
#pragma unroll
                for (int i = 0; i < 8; ++i) squares = __fmaf_rn(v[c][i], v[c][i], squares);
            }
        }
        squares = warp_sum(squares);
        const float inverse = rsqrtf(__fadd_rn(__fdiv_rn(squares, static_cast<float>(D)), eps));
        float absmax = 0.0f;
#pragma unroll
        for (int c = 0; c < CHUNKS; ++c) {
            const int col = (c * 32 + lane) * 8;
            if (col < D) {
                float g[8];
                unpack8(raw_gain[c], g);
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    v[c][i] = __fmul_rn(__fmul_rn(v[c][i], inverse), g[i]);
                    absmax = fmaxf(absmax, fabsf(v[c][i]));
                }
            }
        }
        absmax = fmaxf(warp_max(absmax), 1e-20f);
        const float step_inverse = __fdiv_rn(127.0f, absmax);
#pragma unroll
        for (int c = 0; c < CHUNKS; ++c) {
            const int col = (c * 32 + lane) * 8;
            if (col < D) {
                uint32_t packed[2] = {0u, 0u};
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const int value = __float2int_rn(__fmul_rn(v[c][i], step_inverse));
                    packed[i / 4] |= (static_cast<uint32_t>(value) & 0xffu) << (8 * (i % 4));
                }
                *reinterpret_cast<uint2*>(q + base + col) = make_uint2(packed[0], packed[1]);
            }
        }
        if (lane == 0) scale[row] = __fdiv_rn(absmax, 127.0f);
    }
}

template <int CHUNKS>
__global__ void __launch_bounds__(kRowWarps * 32) rms_norm_kernel(const uint16_t* __restrict__ x, const uint16_t* __restrict__ gain, float eps,
                                                                  uint16_t* __restrict__ y, int M, int D) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row = blockIdx.x * kRowWarps + warp;
    if (row >= M) return;
    const size_t base = static_cast<size_t>(row) * D;
    float v[CHUNKS][8], g[CHUNKS][8];
    float squares = 0.0f;
#pragma unroll
    for (int c = 0; c < CHUNKS; ++c) {
        const int col = (c * 32 + lane) * 8;
        if (col < D) {
            unpack8(*reinterpret_cast<const uint4*>(x + base + col), v[c]);
            unpack8(*reinterpret_cast<const uint4*>(gain + col), g[c]);
#pragma unroll
            for (int i = 0; i < 8; ++i) squares = __fmaf_rn(v[c][i], v[c][i], squares);
        }
    }
    squares = warp_sum(squares);
    const float inverse = rsqrtf(__fadd_rn(__fdiv_rn(squares, static_cast<float>(D)), eps));
#pragma unroll
    for (int c = 0; c < CHUNKS; ++c) {
        const int col = (c * 32 + lane) * 8;
        if (col < D) {
            uint16_t packed[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) packed[i] = f2h_bits(__fmul_rn(__fmul_rn(v[c][i], inverse), g[c][i]));
            *reinterpret_cast<uint4*>(y + base + col) = *reinterpret_cast<const uint4*>(packed);
        }
    }
}

// h [M, hidden] fp16 -> q [M, width] int8 (width <= 1024, a multiple of 32), scale [M]. Lane l of part p owns the
// 8-element chunk c = 32 p + l (coalesced 16-byte loads and 8-byte stores); a Hadamard block of 32 is the chunks of
// 4 consecutive lanes. With i = 8 q + r (q the chunk within the block, r the element within the chunk),
// H32[i][j] = (-1)^popcount(i & j) = H4[q_i][q_j] H8[r_i][r_j]: the butterflies over r run in registers, those over q
// across the quad by shuffles, in the same order over the index bits as a 32-element butterfly.
// A warp takes kRotateRows consecutive rows, their loads all issued first.
constexpr int kRotateRows = 2;
__global__ void __launch_bounds__(kRowWarps * 32) rotate_quant_kernel(const uint16_t* __restrict__ h, int8_t* __restrict__ q,
                                                                      float* __restrict__ scale, int M, int hidden, int width) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int first_row = (blockIdx.x * kRowWarps + warp) * kRotateRows;
    if (first_row >= M) return;
    uint4 raw[kRotateRows][4];
#pragma unroll
    for (int r = 0; r < kRotateRows; ++r)
#pragma unroll
        for (int part = 0; part < 4; ++part) {
            const int col = (part * 32 + lane) * 8;
            raw[r][part] = (col < hidden && first_row + r < M)
                               ? *reinterpret_cast<const uint4*>(h + static_cast<size_t>(first_row + r) * hidden + col)
                               : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
    for (int r = 0; r < kRotateRows; ++r) {
        const int row = first_row + r;
        if (row >= M) break;  // uniform across the warp
        float v[4][8];
#pragma unroll
        for (int part = 0; part < 4; ++part) unpack8(raw[r][part], v[part]);
        // (a, b) -> (a + b, a - b) over the element bits (registers), then over the chunk bits (the quad's lanes)
#pragma unroll
        for (int part = 0; part < 4; ++part) {
#pragma unroll
            for (int span = 1; span < 8; span <<= 1)
#pragma unroll
                for (int i = 0; i < 8; ++i)
                    if ((i & span) == 0) {
                        const float a = v[part][i], b = v[part][i + span];
                        v[part][i] = __fadd_rn(a, b);
                        v[part][i + span] = __fsub_rn(a, b);
                    }
#pragma unroll
            for (int span = 1; span < 4; span <<= 1)
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const float partner = __shfl_xor_sync(0xffffffffu, v[part][i], span);
                    v[part][i] = (lane & span) ? __fsub_rn(partner, v[part][i]) : __fadd_rn(v[part][i], partner);
                }
        }
        float absmax = 0.0f;
#pragma unroll
        for (int part = 0; part < 4; ++part)
#pragma unroll
            for (int i = 0; i < 8; ++i) absmax = fmaxf(absmax, fabsf(v[part][i]));
        absmax = fmaxf(warp_max(absmax), 1e-20f);
        const float step_inverse = __fdiv_rn(127.0f, absmax);
#pragma unroll
        for (int part = 0; part < 4; ++part) {
            const int col = (part * 32 + lane) * 8;
            if (col < width) {
                uint32_t packed[2] = {0u, 0u};
#pragma unroll
                for (int i = 0; i < 8; ++i)
                    packed[i / 4] |= (static_cast<uint32_t>(__float2int_rn(__fmul_rn(v[part][i], step_inverse))) & 0xffu) << (8 * (i % 4));
                *reinterpret_cast<uint2*>(q + static_cast<size_t>(row) * width + col) = make_uint2(packed[0], packed[1]);
            }
        }
        if (lane == 0) scale[row] = __fdiv_rn(absmax, 127.0f);
    }
}

// ---- embedding ------------------------------------------------------------------------------------------------

constexpr int kTokens = 70, kSquares = 64, kFeatures = 23, kVocab = 81, kPieceCodes = 13, kEdge = 13, kNoPiece = 225;
// each feature's first row in the table: 4 x 226 offsets, 8 x 14 neighbours, 8 x 85 lines, 9 knights, 2 x 15 pawns
__constant__ int kFeatureRowOffset[kFeatures] = {0,    226,  452,  678,  904,  918,  932,  946,  960,  974,  988,  1002,
                                                 1016, 1101, 1186, 1271, 1356, 1441, 1526, 1611, 1696, 1705, 1720};
__constant__ int kDirections[8][2] = {{0, 1}, {0, -1}, {1, 0}, {-1, 0}, {1, 1}, {-1, 1}, {1, -1}, {-1, -1}};
__constant__ int kKnightJumps[8][2] = {{1, 2}, {2, 1}, {2, -1}, {1, -2}, {-1, -2}, {-2, -1}, {-2, 1}, {-1, 2}};

FRY_DEVICE int code_at(const int* codes, int file, int rank) {
    return (file >= 0 && file < 8 && rank >= 0 && rank < 8) ? codes[rank * 8 + file] : kEdge;
}

// One CTA per (board, 256 columns): the 64 x 23 feature rows into shared memory, then every (token, 8 columns) summed.
__global__ void __launch_bounds__(256) embedding_kernel(const int64_t* __restrict__ boards, const uint16_t* __restrict__ embed,
                                                        const uint16_t* __restrict__ position, const uint16_t* __restrict__ table,
                                                        uint16_t* __restrict__ out, int D) {
    __shared__ int codes[kTokens];
    __shared__ int firsts[4];
    __shared__ int rows[kSquares][kFeatures];
    const int b = blockIdx.x, tid = threadIdx.x;
    for (int t = tid; t < kTokens; t += blockDim.x) {
        const int64_t token = boards[static_cast<size_t>(b) * kTokens + t];
        const bool ok = t < kSquares ? (token >= 0 && token < kPieceCodes) : (token >= 0 && token < kVocab);
        if (!ok) record_error(kBadToken, b);
        codes[t] = ok ? static_cast<int>(token) : 0;
    }
    __syncthreads();
    if (tid < 4) {
        const int wanted[4] = {6, 12, 5, 11};  // our king, their king, our queen, their queen
        int first = kSquares;
        for (int s = 0; s < kSquares; ++s)
            if (codes[s] == wanted[tid]) {
                first = s;
                break;
            }
        firsts[tid] = first;
    }
    __syncthreads();
    {
        const int s = tid & 63, part = tid >> 6, file = s & 7, rank = s >> 3;
        int* r = rows[s];
        if (part == 0) {
            for (int i = 0; i < 4; ++i) {
                const int p = firsts[i];
                r[i] = kFeatureRowOffset[i] + (p < kSquares ? (rank - (p >> 3) + 7) * 15 + file - (p & 7) + 7 : kNoPiece);
            }
            int ours = 0, theirs = 0;
            for (int j = 0; j < 8; ++j) {
                const int c = code_at(codes, file + kKnightJumps[j][0], rank + kKnightJumps[j][1]);
                ours += c == 2;
                theirs += c == 8;
            }
            r[20] = kFeatureRowOffset[20] + min(ours, 2) * 3 + min(theirs, 2);
        } else if (part == 1) {
            for (int d = 0; d < 8; ++d) r[4 + d] = kFeatureRowOffset[4 + d] + code_at(codes, file + kDirections[d][0], rank + kDirections[d][1]);
        } else if (part == 2) {
            for (int d = 0; d < 8; ++d) {
                int line = 0;
                for (int k = 1; k <= 7; ++k) {
                    const int c = code_at(codes, file + kDirections[d][0] * k, rank + kDirections[d][1] * k);
                    if (c == kEdge) break;
                    if (c != 0) {
                        line = 1 + (c - 1) * 7 + (k - 1);
                        break;
                    }
                }
                r[12 + d] = kFeatureRowOffset[12 + d] + line;
            }
        } else {
            for (int d = 0; d < 2; ++d) {  // up and down the file: the nearest pawn of either side, others do not block
                int pawn = 0;
                for (int k = 1; k <= 7; ++k) {
                    const int c = code_at(codes, file, rank + kDirections[d][1] * k);
                    if (c == kEdge) break;
                    if (c == 1 || c == 7) {
                        pawn = 1 + (c == 7) * 7 + (k - 1);
                        break;
                    }
                }
                r[21 + d] = kFeatureRowOffset[21 + d] + pawn;
            }
        }
    }
    __syncthreads();
    // this CTA's slice of the columns: [blockIdx.y * 256, + 256)
    const int first = blockIdx.y * 256, width = D - first < 256 ? D - first : 256;
    const int vectors = width / 8;
    for (int idx = tid; idx < kTokens * vectors; idx += blockDim.x) {
        const int t = idx / vectors, col = first + (idx % vectors) * 8;
        float e[8], p[8];
        unpack8(*reinterpret_cast<const uint4*>(embed + static_cast<size_t>(codes[t]) * D + col), e);
        unpack8(*reinterpret_cast<const uint4*>(position + static_cast<size_t>(t) * D + col), p);
        float features[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        if (t < kSquares) {
            // all 23 rows in flight before the first add; the adds keep the feature order
            uint4 raw[kFeatures];
#pragma unroll
            for (int f = 0; f < kFeatures; ++f) raw[f] = *reinterpret_cast<const uint4*>(table + static_cast<size_t>(rows[t][f]) * D + col);
#pragma unroll
            for (int f = 0; f < kFeatures; ++f) {
                float row[8];
                unpack8(raw[f], row);
#pragma unroll
                for (int i = 0; i < 8; ++i) features[i] = __fadd_rn(features[i], row[i]);
            }
        }
        uint16_t packed[8];
#pragma unroll
        for (int i = 0; i < 8; ++i)
            packed[i] = f2h_bits(__fadd_rn(__fadd_rn(e[i], p[i]), h2f_bits(f2h_bits(features[i]))));
        *reinterpret_cast<uint4*>(out + (static_cast<size_t>(b) * kTokens + t) * D + col) = *reinterpret_cast<const uint4*>(packed);
    }
}

// ---- launchers ------------------------------------------------------------------------------------------------

cudaError_t norm_quant(const uint16_t* x, const uint16_t* original, const uint16_t* residual_scale, const uint16_t* input_scale,
                       const uint16_t* gain, float eps, uint16_t* mixed, int8_t* q, float* scale, int M, int D, cudaStream_t stream) {
    if (M <= 0) return cudaSuccess;
    if (D % 8 != 0 || D > 1024) return cudaErrorInvalidValue;
    constexpr int kRows = 4, kMixRows = 2;  // rows a warp
    const bool mix = original != nullptr;
    const dim3 grid((M + kRowWarps * (mix ? kMixRows : kRows) - 1) / (kRowWarps * (mix ? kMixRows : kRows)));
    const int chunks = (D + 255) / 256;
#define FRY_NQ(C)                                                                                                                       \
    (mix ? (norm_quant_kernel<C, true, kMixRows><<<grid, kRowWarps * 32, 0, stream>>>(x, original, residual_scale, input_scale, gain, \
                                                                                       eps, mixed, q, scale, M, D), 0)                  \
         : (norm_quant_kernel<C, false, kRows><<<grid, kRowWarps * 32, 0, stream>>>(x, original, residual_scale, input_scale, gain, eps, \
                                                                                     mixed, q, scale, M, D), 0))
    switch (chunks) {
        case 1: FRY_NQ(1); break;
        case 2: FRY_NQ(2); break;
        case 3: FRY_NQ(3); break;
        default: FRY_NQ(4); break;
    }
#undef FRY_NQ
    return cudaGetLastError();
}

cudaError_t rms_norm_f16(const uint16_t* x, const uint16_t* gain, float eps, uint16_t* y, int M, int D, cudaStream_t stream) {
    if (M <= 0) return cudaSuccess;
    if (D % 8 != 0 || D > 1024) return cudaErrorInvalidValue;
    const dim3 grid((M + kRowWarps - 1) / kRowWarps);
    switch ((D + 255) / 256) {
        case 1: rms_norm_kernel<1><<<grid, kRowWarps * 32, 0, stream>>>(x, gain, eps, y, M, D); break;
        case 2: rms_norm_kernel<2><<<grid, kRowWarps * 32, 0, stream>>>(x, gain, eps, y, M, D); break;
        case 3: rms_norm_kernel<3><<<grid, kRowWarps * 32, 0, stream>>>(x, gain, eps, y, M, D); break;
        default: rms_norm_kernel<4><<<grid, kRowWarps * 32, 0, stream>>>(x, gain, eps, y, M, D); break;
    }
    return cudaGetLastError();
}

cudaError_t rotate_quant(const uint16_t* h, int8_t* q, float* scale, int M, int hidden, int width, cudaStream_t stream) {
    if (M <= 0) return cudaSuccess;
    if (hidden % 8 != 0 || width % 32 != 0 || width > 1024 || hidden > width) return cudaErrorInvalidValue;
    const int rows_a_block = kRowWarps * kRotateRows;
    rotate_quant_kernel<<<(M + rows_a_block - 1) / rows_a_block, kRowWarps * 32, 0, stream>>>(h, q, scale, M, hidden, width);
    return cudaGetLastError();
}

cudaError_t board_embedding(const int64_t* boards, const uint16_t* embed, const uint16_t* position, const uint16_t* table,
                            uint16_t* out, int B, int D, cudaStream_t stream) {
    if (B <= 0) return cudaSuccess;
    if (D % 8 != 0) return cudaErrorInvalidValue;
    embedding_kernel<<<dim3(B, (D + 255) / 256), 256, 0, stream>>>(boards, embed, position, table, out, D);
    return cudaGetLastError();
}

}  // namespace fry
