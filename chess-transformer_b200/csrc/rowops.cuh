// One activation row on one warp: the per-row arithmetic of `norm_quant` / `mix_norm_quant`
// (model/int8_blocks.py:156-212) and `rotate_quant` (model/int8_blocks.py:216-251), shared by the standalone row kernels
// (rows.cu) and the GEMM's row-block tails (gemm.cu), so both give the same bits.
//
// Layout: lane l of chunk c owns the 8 columns (32 c + l) * 8 .. +7 of the row (16-byte loads, 8-byte int8 stores).
#pragma once

#include "common.cuh"

namespace fry {

FRY_DEVICE void unpack8(const uint4& u, float (&v)[8]) {
    const uint16_t* h = reinterpret_cast<const uint16_t*>(&u);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = h2f_exact(h[i]);
}

// The gain's values at this lane's columns of each chunk (zero past `width`), unpacked once for every row a warp takes
// where registers allow; norm_quant_row also takes the packed fp16 chunks (load_row_chunks) and unpacks them per row.
template <int CHUNKS>
FRY_DEVICE void load_gain(const uint16_t* gain, int width, int lane, float (&to)[CHUNKS][8]) {
#pragma unroll
    for (int c = 0; c < CHUNKS; ++c) {
        const int col = (c * 32 + lane) * 8;
        unpack8(col < width ? *reinterpret_cast<const uint4*>(gain + col) : make_uint4(0, 0, 0, 0), to[c]);
    }
}

// The row's fp16 chunks of this lane, zero past `width` columns; STREAM: read once, so loaded evict-first (ld.global.cs).
template <int CHUNKS, bool STREAM = false>
FRY_DEVICE void load_row_chunks(const uint16_t* row, int width, int lane, uint4 (&to)[CHUNKS]) {
#pragma unroll
    for (int c = 0; c < CHUNKS; ++c) {
        const int col = (c * 32 + lane) * 8;
        const uint4* at = reinterpret_cast<const uint4*>(row + col);
        to[c] = col < width ? (STREAM ? __ldcs(at) : *at) : make_uint4(0, 0, 0, 0);
    }
}

// rint(v * step) for 8 values (|v * step| < 2^22) as 8 int8 bytes. The product, rounded to fp32, plus 1.5 * 2^23 lands
// in [2^23, 2^24), where the fp32 spacing is 1, so the add's round-to-nearest-even leaves rint(product) in the low
// mantissa bits: the sum's low byte is rint(product) mod 256, the int8 byte. An add, not an fma, so the product is
// rounded first, as __float2int_rn(product) rounds it; and no conversion unit.
FRY_DEVICE uint2 quantize8(const float (&v)[8], float step) {
    const uint64_t step2 = pair2(step, step), magic2 = pair2(12582912.0f, 12582912.0f);
    uint32_t q[8];
#pragma unroll
    for (int i = 0; i < 8; i += 2) {
        const float2 shifted = lanes(add2(mul2(pair2(v[i], v[i + 1]), step2), magic2));
        q[i] = __float_as_uint(shifted.x);
        q[i + 1] = __float_as_uint(shifted.y);
    }
    uint32_t words[2];
#pragma unroll
    for (int w = 0; w < 2; ++w) {
        const uint32_t low = __byte_perm(q[4 * w], q[4 * w + 1], 0x0040), high = __byte_perm(q[4 * w + 2], q[4 * w + 3], 0x0040);
        words[w] = __byte_perm(low, high, 0x5410);
    }
    return make_uint2(words[0], words[1]);
}

// Where norm_quant_row puts a row's int8 values: a plain row in global memory...
struct RowOut {
    int8_t* q;
    FRY_DEVICE void put8(int col, uint2 bytes) const { *reinterpret_cast<uint2*>(q + col) = bytes; }
};
// ...or row r of a K-major int8 operand resident in shared memory as the MMA reads it: 128-byte K slices of 128 rows
// (16 KB each) in the 128-byte swizzle, 16-byte unit u of row r at u ^ (r % 8).
struct SwizzledRowOut {
    uint8_t* tile;
    int row;
    FRY_DEVICE void put8(int col, uint2 bytes) const {
        uint8_t* slice = tile + (col >> 7) * (128 * 128) + row * 128;
        const int unit = (col & 127) >> 4;
        *reinterpret_cast<uint2*>(slice + ((unit ^ (row & 7)) << 4) + (col & 15)) = bytes;
    }
};

// norm_quant of one row of D columns (D <= 256 CHUNKS): x (and with MIX, original: the row first becomes
// fp16(fma(rs, x, is * original)), stored to mixed) -> RMSNorm with gain in fp32 -> int8 by round-half-even into q,
// absmax / 127 into *scale. Arithmetic order: per lane over its chunks, then the warp's tree.
FRY_DEVICE void gain_chunk(const uint4& packed, float (&to)[8]) { unpack8(packed, to); }
FRY_DEVICE void gain_chunk(const float (&values)[8], float (&to)[8]) {
#pragma unroll
    for (int i = 0; i < 8; ++i) to[i] = values[i];
}

template <int CHUNKS, bool MIX, typename Out = RowOut, typename GainChunk>
FRY_DEVICE void norm_quant_row(const uint4 (&raw)[CHUNKS], const uint4 (&raw_original)[MIX ? CHUNKS : 1], const GainChunk (&gain)[CHUNKS],
                               uint64_t rs2, uint64_t is2, float eps, int D, int lane, uint16_t* mixed, const Out& q, float* scale) {
    float v[CHUNKS][8];
    float squares = 0.0f;
#pragma unroll
    for (int c = 0; c < CHUNKS; ++c) {
        const int col = (c * 32 + lane) * 8;
        unpack8(raw[c], v[c]);
        if (col < D) {
            if constexpr (MIX) {
                float o[8];
                unpack8(raw_original[c], o);
                uint32_t packed[4];
#pragma unroll
                for (int i = 0; i < 8; i += 2) {
                    const float2 m = lanes(fma2(rs2, pair2(v[c][i], v[c][i + 1]), mul2(is2, pair2(o[i], o[i + 1]))));
                    packed[i / 2] = pack_half2_rn(m.x, m.y);
                    v[c][i] = h2f_exact(static_cast<uint16_t>(packed[i / 2] & 0xffff));
                    v[c][i + 1] = h2f_exact(static_cast<uint16_t>(packed[i / 2] >> 16));
                }
                *reinterpret_cast<uint4*>(mixed + col) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) squares = __fmaf_rn(v[c][i], v[c][i], squares);
        }
    }
    squares = warp_sum(squares);
    const float inverse = rsqrtf(__fadd_rn(__fdiv_rn(squares, static_cast<float>(D)), eps));
    const uint64_t inverse2 = pair2(inverse, inverse);
    float absmax = 0.0f;
#pragma unroll
    for (int c = 0; c < CHUNKS; ++c) {
        const int col = (c * 32 + lane) * 8;
        if (col < D) {
            float g[8];
            gain_chunk(gain[c], g);
#pragma unroll
            for (int i = 0; i < 8; i += 2) {
                const float2 y = lanes(mul2(mul2(pair2(v[c][i], v[c][i + 1]), inverse2), pair2(g[i], g[i + 1])));
                v[c][i] = y.x;
                v[c][i + 1] = y.y;
                absmax = fmaxf(absmax, fmaxf(fabsf(y.x), fabsf(y.y)));
            }
        }
    }
    absmax = fmaxf(warp_max_redux(absmax), 1e-20f);
    const float step_inverse = __fdiv_rn(127.0f, absmax);
#pragma unroll
    for (int c = 0; c < CHUNKS; ++c) {
        const int col = (c * 32 + lane) * 8;
        if (col < D) q.put8(col, quantize8(v[c], step_inverse));
    }
    if (lane == 0) *scale = __fdiv_rn(absmax, 127.0f);
}

// rotate_quant of one row: h (fp16, hidden columns, zero beyond) -> times the block-diagonal 32x32 Sylvester Hadamard
// matrix -> int8 by round-half-even into q (width <= 1024 columns, a multiple of 32), absmax / 127 into *scale.
// A Hadamard block of 32 is the chunks of 4 consecutive lanes. With i = 8 q + r (q the chunk within the block, r the
// element within the chunk), H32[i][j] = (-1)^popcount(i & j) = H4[q_i][q_j] H8[r_i][r_j]: the butterflies over r run in
// registers, those over q across the quad by shuffles, in the same order over the index bits as a 32-element butterfly.
FRY_DEVICE void rotate_quant_row(const uint4 (&raw)[4], int width, int lane, int8_t* q, float* scale) {
    float v[4][8];
#pragma unroll
    for (int part = 0; part < 4; ++part) unpack8(raw[part], v[part]);
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
    absmax = fmaxf(warp_max_redux(absmax), 1e-20f);
    const float step_inverse = __fdiv_rn(127.0f, absmax);
#pragma unroll
    for (int part = 0; part < 4; ++part) {
        const int col = (part * 32 + lane) * 8;
        if (col < width) *reinterpret_cast<uint2*>(q + col) = quantize8(v[part], step_inverse);
    }
    if (lane == 0) *scale = __fdiv_rn(absmax, 127.0f);
}

}  // namespace fry
