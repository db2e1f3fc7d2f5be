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
#include "rowops.cuh"

namespace fry {

constexpr int kRowWarps = 8;
constexpr int kRowCtasPerSm = 3;  // persistent row kernels: CTAs of kRowWarps warps an SM
// from kMidRows up to kLargeRows rows the persistent row kernels take more, smaller CTAs, more warps an SM: at 64 boards
// (4480 rows) rotate_quant 4.90 -> 4.2 us and norm_quant 3.80 -> 3.63 us a launch, the forward 1.844 -> 1.823 ms; at
// 16 boards the forward was 2.6% slower that way, and at 256 boards 8 x 3 stays best or level
constexpr int kSmallRowWarps = 4, kSmallRowCtasPerSm = 7, kMidRows = 4096, kLargeRows = 8192;
inline bool mid_rows(int M) { return M >= kMidRows && M < kLargeRows; }

// x [M, D] fp16 -> q [M, D] int8, scale [M]; with MIX, x is first mixed with original and the mix stored to mixed.
// Persistent warps: warp w of W takes rows w, w + W, ..., loading the next row while it works on this one. A row's
// arithmetic is the single-row order: per lane over its chunks, then the warp's tree.
template <int CHUNKS, bool MIX, int WARPS = kRowWarps, int CTAS = kRowCtasPerSm>
__global__ void __launch_bounds__(WARPS * 32, CTAS) norm_quant_kernel(const uint16_t* __restrict__ x, const uint16_t* __restrict__ original,
                                                                    const uint16_t* residual_scale, const uint16_t* input_scale,
                                                                    const uint16_t* __restrict__ gain, float eps, uint16_t* mixed,
                                                                    int8_t* __restrict__ q, float* __restrict__ scale, int M, int D) {
    grid_dependency_start();
    const int lane = threadIdx.x & 31;
    const int stride = gridDim.x * WARPS;
    int row = blockIdx.x * WARPS + (threadIdx.x >> 5);
    if (row >= M) return;
    float rs = 0.0f, is = 0.0f;
    if constexpr (MIX) {
        rs = h2f_bits(*residual_scale);
        is = h2f_bits(*input_scale);
    }
    const uint64_t rs2 = pair2(rs, rs), is2 = pair2(is, is);
    uint4 raw_gain[CHUNKS], raw[CHUNKS], raw_original[MIX ? CHUNKS : 1];
    auto load_row = [&](int r, uint4 (&to)[CHUNKS], uint4 (&to_original)[MIX ? CHUNKS : 1]) {
#pragma unroll
        for (int c = 0; c < CHUNKS; ++c) {
            const int col = (c * 32 + lane) * 8;
            const size_t at = static_cast<size_t>(r) * D + col;
            to[c] = col < D ? *reinterpret_cast<const uint4*>(x + at) : make_uint4(0, 0, 0, 0);
            if constexpr (MIX) to_original[c] = col < D ? *reinterpret_cast<const uint4*>(original + at) : make_uint4(0, 0, 0, 0);
        }
    };
    load_row_chunks<CHUNKS>(gain, D, lane, raw_gain);  // packed: the unpacked gain would not fit 3 CTAs an SM
    load_row(row, raw, raw_original);
    for (; row < M; row += stride) {  // uniform across the warp
        uint4 next[CHUNKS], next_original[MIX ? CHUNKS : 1];
        if (row + stride < M) load_row(row + stride, next, next_original);
        const size_t base = static_cast<size_t>(row) * D;
        norm_quant_row<CHUNKS, MIX>(raw, raw_original, raw_gain, rs2, is2, eps, D, lane, mixed + base, RowOut{q + base}, scale + row);
#pragma unroll
        for (int c = 0; c < CHUNKS; ++c) {
            raw[c] = next[c];
            if constexpr (MIX) raw_original[c] = next_original[c];
        }
    }
}

template <int CHUNKS>
__global__ void __launch_bounds__(kRowWarps * 32) rms_norm_kernel(const uint16_t* __restrict__ x, const uint16_t* __restrict__ gain, float eps,
                                                                  uint16_t* __restrict__ y, int M, int D) {
    grid_dependency_start();
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

// h [M, hidden] fp16 -> q [M, width] int8 (width <= 1024, a multiple of 32), scale [M], by rotate_quant_row.
// Persistent warps, as norm_quant: warp w of W takes rows w, w + W, ..., loading the next row while it works on one.
template <int WARPS = kRowWarps, int CTAS = kRowCtasPerSm>
__global__ void __launch_bounds__(WARPS * 32, CTAS) rotate_quant_kernel(const uint16_t* __restrict__ h, int8_t* __restrict__ q,
                                                                        float* __restrict__ scale, int M, int hidden, int width) {
    grid_dependency_start();
    const int lane = threadIdx.x & 31;
    const int stride = gridDim.x * WARPS;
    int row = blockIdx.x * WARPS + (threadIdx.x >> 5);
    if (row >= M) return;
    uint4 raw[4];
    load_row_chunks<4, true>(h + static_cast<size_t>(row) * hidden, hidden, lane, raw);
    for (; row < M; row += stride) {  // uniform across the warp
        uint4 next[4];
        if (row + stride < M) load_row_chunks<4, true>(h + static_cast<size_t>(row + stride) * hidden, hidden, lane, next);
        rotate_quant_row(raw, width, lane, q + static_cast<size_t>(row) * width, scale + row);
#pragma unroll
        for (int c = 0; c < 4; ++c) raw[c] = next[c];
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

// A board's tokens into codes[70] (a token outside the vocabulary read as 0 and recorded), the squares of our king,
// their king, our queen and their queen into firsts[4] (64: none), and each square's 23 feature rows of the table, each
// feature's first row added (SquareFeatures.indices, model/model.py:134-169), into rows[64][23]. A board's tokens:
// int64 [70] (boards, pitch 70) or the first 70 bytes of a lean lane's row (pitch kLeanRow). All 256 threads of the
// CTA call it; it ends with the rows written but not yet synchronised.
template <typename Token>
FRY_DEVICE void board_feature_rows(const Token* __restrict__ boards, int pitch, int b, int* codes, int* firsts, int (*rows)[kFeatures],
                                   int tid) {
    for (int t = tid; t < kTokens; t += blockDim.x) {
        const int64_t token = static_cast<int64_t>(boards[static_cast<size_t>(b) * pitch + t]);
        const bool ok = t < kSquares ? (token >= 0 && token < kPieceCodes) : (token >= 0 && token < kVocab);
        if (!ok) record_error(kBadToken, b);
        codes[t] = ok ? static_cast<int>(token) : 0;
    }
    __syncthreads();
    if (tid < 32) {  // the first square of our king, their king, our queen, their queen: a warp's ballots over the squares
        const int wanted[4] = {6, 12, 5, 11};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const unsigned low = __ballot_sync(0xffffffffu, codes[tid] == wanted[i]), high = __ballot_sync(0xffffffffu, codes[32 + tid] == wanted[i]);
            if (tid == 0) firsts[i] = low ? __ffs(low) - 1 : high ? 32 + __ffs(high) - 1 : kSquares;
        }
    }
    __syncthreads();
    {
        // four threads a square, the walks along lines shared out so no thread takes more than about 28 lookups
        const int s = tid & 63, part = tid >> 6, file = s & 7, rank = s >> 3;
        int* r = rows[s];
        // the nearest piece along direction d: 1 + (code - 1) * 7 + (distance - 1), 0 if none before the edge
        auto line_row = [&](int d) {
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
        };
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
            line_row(0);
            line_row(1);
        } else if (part == 2) {
            for (int d = 2; d < 6; ++d) line_row(d);
        } else {
            line_row(6);
            line_row(7);
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
}

// One CTA per (board, slice of `slice` columns, group of tokens): the 64 x 23 feature rows into shared memory, then
// every (token, 8 columns) of its share summed. Small batches split a board's tokens over more CTAs (gridDim.z), so
// each thread's chain of gathers is short.
template <typename Token>
__global__ void __launch_bounds__(256) embedding_kernel(const Token* __restrict__ boards, int pitch, const uint16_t* __restrict__ embed,
                                                        const uint16_t* __restrict__ position, const uint16_t* __restrict__ table,
                                                        uint16_t* __restrict__ out, int D, int slice) {
    grid_dependency_start();
    __shared__ int codes[kTokens];
    __shared__ int firsts[4];
    __shared__ int rows[kSquares][kFeatures];
    const int b = blockIdx.x, tid = threadIdx.x;
    board_feature_rows(boards, pitch, b, codes, firsts, rows, tid);
    __syncthreads();
    // this CTA's slice of the columns, [blockIdx.y * slice, + slice), and its tokens, [token_begin, token_end)
    const int first = blockIdx.y * slice, width = D - first < slice ? D - first : slice;
    const int vectors = width / 8;
    const int token_begin = blockIdx.z * kTokens / gridDim.z, token_end = (blockIdx.z + 1) * kTokens / gridDim.z;
    for (int idx = tid; idx < (token_end - token_begin) * vectors; idx += blockDim.x) {
        const int t = token_begin + idx / vectors, col = first + (idx % vectors) * 8;
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

// One CTA per board: its squares' 23 feature rows, int32 [64, 23] a board (the rows embedding_kernel sums).
__global__ void __launch_bounds__(256) feature_rows_kernel(const int64_t* __restrict__ boards, int32_t* __restrict__ out) {
    grid_dependency_start();
    __shared__ int codes[kTokens];
    __shared__ int firsts[4];
    __shared__ int rows[kSquares][kFeatures];
    const int b = blockIdx.x, tid = threadIdx.x;
    board_feature_rows(boards, kTokens, b, codes, firsts, rows, tid);
    __syncthreads();
    for (int i = tid; i < kSquares * kFeatures; i += blockDim.x) out[static_cast<size_t>(b) * kSquares * kFeatures + i] = rows[i / kFeatures][i % kFeatures];
}

// ---- launchers ------------------------------------------------------------------------------------------------

cudaError_t norm_quant(const uint16_t* x, const uint16_t* original, const uint16_t* residual_scale, const uint16_t* input_scale,
                       const uint16_t* gain, float eps, uint16_t* mixed, int8_t* q, float* scale, int M, int D, cudaStream_t stream) {
    if (M <= 0) return cudaSuccess;
    if (D % 8 != 0 || D > 1024) return cudaErrorInvalidValue;
    const bool mix = original != nullptr;
    // persistent warps: up to kRowCtasPerSm CTAs an SM, each warp looping over rows (kSmallRow* from kMidRows to kLargeRows)
    int device = 0, multiprocessors = 0;
    cudaError_t status = cudaGetDevice(&device);
    if (status == cudaSuccess) status = cudaDeviceGetAttribute(&multiprocessors, cudaDevAttrMultiProcessorCount, device);
    if (status != cudaSuccess) return status;
    const bool small = mid_rows(M);
    const int warps = small ? kSmallRowWarps : kRowWarps, ctas = small ? kSmallRowCtasPerSm : kRowCtasPerSm;
    const int wanted = (M + warps - 1) / warps, most = multiprocessors * ctas;
    const dim3 grid(wanted < most ? wanted : most);
    const int chunks = (D + 255) / 256;
#define FRY_NQ_SHAPE(C, W, N)                                                                                                         \
    status = mix ? launch_dependent(norm_quant_kernel<C, true, W, N>, grid, dim3(W * 32), 0, stream, x, original, residual_scale,     \
                                    input_scale, gain, eps, mixed, q, scale, M, D)                                                    \
                 : launch_dependent(norm_quant_kernel<C, false, W, N>, grid, dim3(W * 32), 0, stream, x, original, residual_scale,    \
                                    input_scale, gain, eps, mixed, q, scale, M, D)
#define FRY_NQ(C)                                                                                                                    \
    if (small) {                                                                                                                     \
        FRY_NQ_SHAPE(C, kSmallRowWarps, kSmallRowCtasPerSm);                                                                        \
    } else {                                                                                                                         \
        FRY_NQ_SHAPE(C, kRowWarps, kRowCtasPerSm);                                                                                  \
    }
    switch (chunks) {
        case 1: FRY_NQ(1); break;
        case 2: FRY_NQ(2); break;
        case 3: FRY_NQ(3); break;
        default: FRY_NQ(4); break;
    }
#undef FRY_NQ_SHAPE
#undef FRY_NQ
    return status;
}

// 8 fp16 values a thread, grid-stride: the three roundings of torch's fp16 `rs * x + is * original`.
__global__ void __launch_bounds__(256) mix_input_f16_kernel(const uint16_t* __restrict__ x, const uint16_t* __restrict__ original,
                                                            const uint16_t* __restrict__ residual_scale, const uint16_t* __restrict__ input_scale,
                                                            uint16_t* out, size_t vectors) {
    grid_dependency_start();
    const float rs = h2f_bits(*residual_scale), is = h2f_bits(*input_scale);
    for (size_t v = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; v < vectors; v += static_cast<size_t>(gridDim.x) * blockDim.x) {
        float a[8], o[8];
        unpack8(reinterpret_cast<const uint4*>(x)[v], a);
        unpack8(reinterpret_cast<const uint4*>(original)[v], o);
        uint32_t words[4];
#pragma unroll
        for (int i = 0; i < 8; i += 2) {
            const uint32_t scaled = pack_half2_rn(__fmul_rn(rs, a[i]), __fmul_rn(rs, a[i + 1]));
            const uint32_t added = pack_half2_rn(__fmul_rn(is, o[i]), __fmul_rn(is, o[i + 1]));
            words[i / 2] = pack_half2_rn(__fadd_rn(h2f_exact(static_cast<uint16_t>(scaled & 0xffff)), h2f_exact(static_cast<uint16_t>(added & 0xffff))),
                                         __fadd_rn(h2f_exact(static_cast<uint16_t>(scaled >> 16)), h2f_exact(static_cast<uint16_t>(added >> 16))));
        }
        reinterpret_cast<uint4*>(out)[v] = make_uint4(words[0], words[1], words[2], words[3]);
    }
}

cudaError_t mix_input_f16(const uint16_t* x, const uint16_t* original, const uint16_t* residual_scale, const uint16_t* input_scale,
                          uint16_t* out, int M, int D, cudaStream_t stream) {
    if (M <= 0) return cudaSuccess;
    if (D % 8 != 0) return cudaErrorInvalidValue;
    const size_t vectors = static_cast<size_t>(M) * D / 8;
    int device = 0, multiprocessors = 0;
    cudaError_t status = cudaGetDevice(&device);
    if (status == cudaSuccess) status = cudaDeviceGetAttribute(&multiprocessors, cudaDevAttrMultiProcessorCount, device);
    if (status != cudaSuccess) return status;
    const size_t wanted = (vectors + 255) / 256, most = static_cast<size_t>(multiprocessors) * 8;
    return launch_dependent(mix_input_f16_kernel, dim3(static_cast<unsigned>(wanted < most ? wanted : most)), dim3(256), 0, stream, x, original,
                            residual_scale, input_scale, out, vectors);
}

cudaError_t rms_norm_f16(const uint16_t* x, const uint16_t* gain, float eps, uint16_t* y, int M, int D, cudaStream_t stream) {
    if (M <= 0) return cudaSuccess;
    if (D % 8 != 0 || D > 1024) return cudaErrorInvalidValue;
    const dim3 grid((M + kRowWarps - 1) / kRowWarps);
    switch ((D + 255) / 256) {
        case 1: return launch_dependent(rms_norm_kernel<1>, grid, dim3(kRowWarps * 32), 0, stream, x, gain, eps, y, M, D);
        case 2: return launch_dependent(rms_norm_kernel<2>, grid, dim3(kRowWarps * 32), 0, stream, x, gain, eps, y, M, D);
        case 3: return launch_dependent(rms_norm_kernel<3>, grid, dim3(kRowWarps * 32), 0, stream, x, gain, eps, y, M, D);
        default: return launch_dependent(rms_norm_kernel<4>, grid, dim3(kRowWarps * 32), 0, stream, x, gain, eps, y, M, D);
    }
}

cudaError_t rotate_quant(const uint16_t* h, int8_t* q, float* scale, int M, int hidden, int width, cudaStream_t stream) {
    if (M <= 0) return cudaSuccess;
    if (hidden % 8 != 0 || width % 32 != 0 || width > 1024 || hidden > width) return cudaErrorInvalidValue;
    int device = 0, multiprocessors = 0;
    cudaError_t status = cudaGetDevice(&device);
    if (status == cudaSuccess) status = cudaDeviceGetAttribute(&multiprocessors, cudaDevAttrMultiProcessorCount, device);
    if (status != cudaSuccess) return status;
    if (mid_rows(M)) {
        const int wanted = (M + kSmallRowWarps - 1) / kSmallRowWarps, most = multiprocessors * kSmallRowCtasPerSm;
        return launch_dependent(rotate_quant_kernel<kSmallRowWarps, kSmallRowCtasPerSm>, dim3(wanted < most ? wanted : most),
                                dim3(kSmallRowWarps * 32), 0, stream, h, q, scale, M, hidden, width);
    }
    const int wanted = (M + kRowWarps - 1) / kRowWarps, most = multiprocessors * kRowCtasPerSm;
    return launch_dependent(rotate_quant_kernel<>, dim3(wanted < most ? wanted : most), dim3(kRowWarps * 32), 0, stream, h, q, scale, M, hidden,
                            width);
}

// The embedding's grid: 256-column slices while the boards give at least two CTAs an SM; below that 128-column slices
// and each board's tokens split over up to 10 CTAs, as many as take the CTAs to two an SM (1 board: 60 CTAs of 7 tokens).
cudaError_t embedding_grid(int B, int D, dim3* grid, int* slice) {
    int device = 0, multiprocessors = 0;
    cudaError_t status = cudaGetDevice(&device);
    if (status == cudaSuccess) status = cudaDeviceGetAttribute(&multiprocessors, cudaDevAttrMultiProcessorCount, device);
    if (status != cudaSuccess) return status;
    const int wanted = 2 * multiprocessors;
    *slice = 256;
    int slices = (D + 255) / 256, groups = 1;
    if (B * slices < wanted) {
        *slice = 128;
        slices = (D + 127) / 128;
        groups = (wanted + B * slices - 1) / (B * slices);
        groups = groups < 1 ? 1 : groups > 10 ? 10 : groups;
    }
    *grid = dim3(B, slices, groups);
    return cudaSuccess;
}

cudaError_t board_embedding(const int64_t* boards, const uint16_t* embed, const uint16_t* position, const uint16_t* table,
                            uint16_t* out, int B, int D, cudaStream_t stream) {
    if (B <= 0) return cudaSuccess;
    if (D % 8 != 0) return cudaErrorInvalidValue;
    dim3 grid;
    int slice = 0;
    const cudaError_t status = embedding_grid(B, D, &grid, &slice);
    if (status != cudaSuccess) return status;
    return launch_dependent(embedding_kernel<int64_t>, grid, dim3(256), 0, stream, boards, kTokens, embed, position, table, out, D, slice);
}

cudaError_t square_feature_rows(const int64_t* boards, int32_t* rows, int B, cudaStream_t stream) {
    if (B <= 0) return cudaSuccess;
    return launch_dependent(feature_rows_kernel, dim3(B), dim3(256), 0, stream, boards, rows);
}

cudaError_t board_embedding_lean(const uint8_t* lean_rows, const uint16_t* embed, const uint16_t* position, const uint16_t* table,
                                 uint16_t* out, int B, int D, cudaStream_t stream) {
    if (B <= 0) return cudaSuccess;
    if (D % 8 != 0) return cudaErrorInvalidValue;
    dim3 grid;
    int slice = 0;
    const cudaError_t status = embedding_grid(B, D, &grid, &slice);
    if (status != cudaSuccess) return status;
    return launch_dependent(embedding_kernel<uint8_t>, grid, dim3(256), 0, stream, lean_rows, kLeanRow, embed, position, table, out, D,
                            slice);
}

}  // namespace fry
