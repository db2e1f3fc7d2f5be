// Tensor-core GEMMs for the Fry forward: out[M, N] = epilogue(A[M, K] . B[N, K]^T) with both operands K-major.
//
//  kind::i8  (int8 x int8 -> int32 in TMEM): the int8 linears of a block (projection, gate_up, down), replacing
//            `int8_linear` (model/int8_blocks.py:66-139) and `small_int8` (model/int8_cuda.py:34-183) of the reference.
//  kind::f16 (fp16 x fp16 -> fp32 in TMEM): `linear` (model/fused_blocks.py:229-318): attention-out (combine_heads,
//            + bias + residual, fp16 out) and the policy head's `a` matmul (+ bias, fp32 out).
//
// A persistent CTA per SM walks its share of the 128 x BN output tiles (tile = blockIdx.x, += gridDim.x). Warp 16
// streams 128-byte-wide K slices of A and B into a ring of shared-memory stages with TMA (128-byte swizzle), running on
// into the next tile; warp 17 issues tcgen05.mma from one elected thread into one of two TMEM accumulators, frees each
// stage with tcgen05.commit and hands the finished accumulator to the epilogue. Warps 0-15 are the epilogue: warp w reads
// TMEM lanes 32 (w % 4) .. +31 (one output row per thread) and every fourth 16-column chunk, starting at chunk w / 4, with
// tcgen05.ld, and applies the epilogue in the reference's op order (model/int8_cuda.py:163-178) while the MMAs of the
// next tile fill the other accumulator.
//
// fp16 outputs leave through shared memory, a sub-tile of SUB columns at a time: staged as 64-column boxes of 128 rows x
// 128 bytes in the 128-byte swizzle (16-byte unit u of row r at u ^ (r % 8), so the 32 rows of a warp's store spread
// over all banks), which warp 18 writes to global memory with TMA stores; no thread stores a row of its own. The row
// operands (residual, original) arrive the same way, as TMA loads of the same boxes that warp 18 issues two sub-tiles
// ahead into one of three slots, and each output overwrites its residual in the slot. A tile's column operands (weight
// scales, bias) are staged one tile ahead in shared memory too, so one barrier a sub-tile suffices.
//
// Normed A (NKS > 0): the int8 A operand is not loaded but made in the prologue of each 128-row block: the epilogue warps
// run norm_quant (rowops.cuh) on the block's fp16 rows straight into NKS resident 128-byte K slices of shared memory,
// in the layout the MMA reads, and the row scales beside them; the CTA then takes every column tile of the block in turn
// while only B streams. The norm's output never reaches global memory.
// CTA pairs (PAIR, the fp16 linear at large M): two CTAs of a cluster share each M = 256 MMA (tcgen05 of the pair
// group). Each loads its 128 rows of A and half of B's rows into its own shared memory; both CTAs' loads complete on
// the even CTA's stage barrier; the even CTA's MMA warp issues the pair's MMAs and commits to the stage and accumulator
// barriers of both CTAs; each CTA's epilogue reads its own TMEM (its 128 rows) and returns the accumulator to the even
// CTA's barrier. A tile is then 256 rows, and each CTA moves half the B bytes.
// No TMA load multicasts.
#include <mutex>
#include <string>

#include "common.cuh"
#include "kernels.h"
#include "rowops.cuh"

namespace fry {

constexpr int kBlockM = 128;
constexpr int kTileKBytes = 128;  // one swizzle row: the K bytes a stage holds
constexpr int kEpilogueWarps = 16;
constexpr int kEpilogueThreads = kEpilogueWarps * 32;
constexpr int kChunkParts = kEpilogueWarps / 4;  // warps sharing one TMEM lane quarter, each taking every kChunkParts-th chunk
constexpr int kProducerWarp = kEpilogueWarps, kMmaWarp = kEpilogueWarps + 1, kStoreWarp = kEpilogueWarps + 2;
constexpr int kGemmThreads = (kEpilogueWarps + 3) * 32;
constexpr int kMmaKBytes = 32;    // K bytes one MMA instruction consumes (32 int8 or 16 fp16)
constexpr int kEpilogueBarrier = 1;  // named barrier of the epilogue warps and the store warp (0 is __syncthreads)
constexpr int kChunkCols = 16;       // columns of one epilogue chunk (one tcgen05.ld)
constexpr int kBoxCols = 64;         // columns of one staged box: 128 bytes of fp16, one swizzle row
constexpr int kBoxBytes = kBlockM * kBoxCols * 2;  // a staged fp16 box: 128 rows x 128 bytes
// dynamic shared memory a CTA may use (227 KB) less the barriers. It starts 1024-byte aligned (after the CTA's 1 KB of
// reserved shared memory), as the 128-byte swizzle atoms need; a kernel checks and records kMisaligned otherwise.
constexpr int kBarrierBytes = 256;
constexpr int kSmemBudget = 227 * 1024 - kBarrierBytes;
constexpr int kNormedK = 768, kNormedSlices = kNormedK / kTileKBytes;  // the one width a normed A is built for
constexpr int kMaxCluster = 4;  // kEpiLinearNorm: CTAs (column tiles) of a row block, one cluster
constexpr int kNormBarrier = 2;  // named barrier of the 16 epilogue warps alone
// fp16 linear epilogues (the bias and the residual optional)
__host__ __device__ constexpr bool linear16(int epi) { return epi == kEpiLinearF16 || epi == kEpiLinearNorm || epi == kEpiMixF16; }
// epilogues that mix the next block's input (residual and original row operands)
__host__ __device__ constexpr bool mixes(int epi) { return epi == kEpiMix || epi == kEpiMixF16; }
// int8 epilogues that scale the sums by the row's activation scale and the column's weight scale
__host__ __device__ constexpr bool scaled(int epi) { return epi <= kEpiMix || epi == kEpiScaleBf16 || epi == kEpiBiasQkNorm; }
// the bias epilogue, with or without the q/k norm after it
__host__ __device__ constexpr bool biased(int epi) { return epi == kEpiBias || epi == kEpiBiasQkNorm; }

// SUB: the columns an epilogue sub-tile stages (whole 64-column boxes, dividing BN); a BN-wide accumulator (one MMA of
// up to N = 256) leaves in BN / SUB sub-tiles, so the staging slots stay small beside the pipeline stages.
template <int KIND, int BN, bool GATED, int EPI, int SUB, int NKS, bool PAIR = false>
struct GemmShape {
    static constexpr int kElem = KIND == 0 ? 1 : 2;
    static constexpr int kBoxK = kTileKBytes / kElem;
    static constexpr int kABytes = kBlockM * kTileKBytes;
    // PAIR (the two CTAs of a cluster share one M = 256 MMA): each holds half of the MMA's B rows, the gate's or the
    // up's when gated
    static constexpr int kBRows = PAIR && !GATED ? BN / 2 : BN;
    static constexpr int kBBytes = kBRows * kTileKBytes;
    // a normed A is resident (NKS slices), so a stage holds B alone
    static constexpr int kResidentBytes = NKS * kABytes;
    static constexpr int kRowScaleBytes = NKS > 0 ? kBlockM * 4 : 0;
    static constexpr int kStageBytes = (NKS > 0 ? 0 : kABytes) + kBBytes * (GATED && !PAIR ? 2 : 1);
    static_assert(!PAIR || (NKS == 0 && EPI != kEpiLinearNorm && kBRows % 8 == 0),
                  "a CTA pair loads its A, has no cluster epilogue and holds B halves of whole 8-row swizzle atoms");
    static_assert(NKS == 0 || (KIND == 0 && NKS * kTileKBytes <= 1024 && NKS % 2 == 0), "a normed A is int8, 256 to 1024 columns");
    // fp16 outputs are staged for TMA stores; int32 and fp32 outputs are stored by their threads
    static constexpr bool kStaged = EPI != kEpiInt32 && EPI != kEpiLinearF32;
    // the epilogue's row operands (residual, and original when mixing), loaded into the staging slots
    static constexpr int kRowTensors = mixes(EPI) ? 2 : (EPI == kEpiResidual || linear16(EPI)) ? 1 : 0;
    // chunks of 16 columns a thread takes in a sub-tile (the 4 warps of a TMEM lane quarter share a sub-tile's chunks)
    static constexpr int kChunksPerSub = SUB / (kChunkCols * kChunkParts) > 0 ? SUB / (kChunkCols * kChunkParts) : 1;
    static constexpr int kSubs = BN / SUB;       // sub-tiles a tile
    static constexpr int kSub = SUB;
    static constexpr int kBoxes = SUB / kBoxCols;  // staged boxes a sub-tile (per row tensor)
    static_assert(!kStaged || (SUB % kBoxCols == 0 && BN % SUB == 0), "a staged sub-tile is whole 64-column boxes");
    static_assert(kStaged || SUB == BN, "unstaged epilogues take the tile whole");
    // one slot holds a sub-tile's row operands (the output overwrites the first) or, without row operands, its output;
    // there are three, so while one is worked on, the next sub-tiles' row operands load two ahead, or (without row
    // operands) the last sub-tile's stores keep reading their slot through the next sub-tile. The normed A and the norm
    // epilogue keep two, which leaves their larger shared-memory residents their pipeline stages.
    static constexpr int kSlotBytes = kStaged ? (kRowTensors > 1 ? kRowTensors : 1) * kBoxes * kBoxBytes : 0;
    // Gated with 128-column sub-tiles (gate_up's pairs) keeps two 32 KB slots too, for a fifth pipeline stage: the
    // forward 4.590 -> 4.572 ms at 256 boards.
    static constexpr int kSlots = (NKS > 0 || EPI == kEpiLinearNorm || (GATED && SUB == 128)) ? 2 : 3;
    static constexpr int kIoBytes = kSlots * kSlotBytes;
    // the tile's column operands, double-buffered by tile: [2][2][BN] floats (weight scales; up's scales or the bias)
    // (the mix and residual epilogues use the scales alone, the fp16 linears the bias alone: one array)
    // (the q/k norm epilogue a third: each column's gain, 0 past the key columns)
    static constexpr int kColumnArrays = EPI == kEpiBiasQkNorm ? 3 : (biased(EPI) || EPI == kEpiGated || EPI == kEpiLinearNorm) ? 2 : 1;
    // kEpiLinearNorm: the cluster's exchange of row partials [2 tiles][kMaxCluster ranks][128 rows][2] and the epilogue
    // warps' own [2][4 parts][128 rows], floats
    static constexpr int kNormBytes = EPI == kEpiLinearNorm ? (2 * kMaxCluster * kBlockM * 2 + 2 * 4 * kBlockM) * 4 : 0;
    static_assert(EPI != kEpiLinearNorm || (KIND == 1 && SUB == 128), "the norm epilogue keeps 4 chunks a thread (fp16 linear, 128-column sub-tiles)");
    static constexpr int kSecond = kColumnArrays >= 2 ? BN : 0;  // where the second operand (up's scales, the bias) starts
    static constexpr int kColumnBytes = 2 * kColumnArrays * BN * 4;
    static constexpr int kStagesFit = (kSmemBudget - kResidentBytes - kRowScaleBytes - kIoBytes - kColumnBytes - kNormBytes) / kStageBytes;
    static constexpr int kStages = kStagesFit > 8 ? 8 : kStagesFit;
    static_assert(kStages >= 2, "at least two pipeline stages");
    static constexpr int kAccCols = BN * (GATED ? 2 : 1);  // one accumulator; two are allocated
    static constexpr int kTmemCols = 2 * kAccCols <= 64 ? 64 : 2 * kAccCols <= 128 ? 128 : 2 * kAccCols <= 256 ? 256 : 512;
    static_assert(2 * kAccCols <= 512, "two accumulators fit TMEM's 512 columns");
    static constexpr int kSmemBytes =
        kResidentBytes + kIoBytes + kStages * kStageBytes + kColumnBytes + kRowScaleBytes + kNormBytes + kBarrierBytes;
    static_assert(kAccCols % 16 == 0 && kAccCols >= 16 && kAccCols <= 256, "an M=128 MMA takes N in steps of 16 up to 256");
    static_assert(kABytes % 1024 == 0 && kBBytes % 1024 == 0, "stages stay 1024-byte aligned for the swizzle atoms");
};

FRY_DEVICE void epilogue_sync() { asm volatile("bar.sync %0, %1;" ::"n"(kEpilogueBarrier), "n"(kEpilogueThreads + 32) : "memory"); }

// A tile's column operands for one column n, as loaded: the weight scale (scaled epilogues), up's weight scale (gated)
// or the fp32 bias, the fp16 bias, and the fp16 gain (the norm epilogue's, or the q/k norm's for a query or key column);
// zero past N. They are loaded a tile ahead into registers and written to shared memory at the end of that tile (by
// store_columns), so the loads' latency passes while the thread works on the tile before.
struct ColumnLoad {
    float scale = 0.0f, second = 0.0f;
    uint16_t half = 0, gain = 0;  // fp16 bits; zero bits are +0.0
};
template <int EPI>
FRY_DEVICE ColumnLoad load_columns(const GemmArgs& p, int n, int N) {
    ColumnLoad c;
    const bool ok = n < N;
    if constexpr (scaled(EPI)) c.scale = ok ? p.w_scale[n] : 0.0f;
    if constexpr (EPI == kEpiGated) c.second = ok ? p.w_scale[N + n] : 0.0f;
    if constexpr (EPI == kEpiLinearF32) c.second = (ok && p.bias_f32) ? p.bias_f32[n] : 0.0f;
    if constexpr (biased(EPI) || linear16(EPI) || EPI == kEpiGatedF16) c.half = (ok && p.bias) ? p.bias[n] : 0;
    if constexpr (EPI == kEpiLinearNorm) c.gain = (ok && p.norm_gain) ? p.norm_gain[n] : 0;
    if constexpr (EPI == kEpiBiasQkNorm) {
        if (n < p.qk_queries) c.gain = p.q_gain[n % p.qk_dq];
        else if (n < p.qk_keys) c.gain = p.k_gain[(n - p.qk_queries) % p.qk_dq];
    }
    return c;
}
// Column i's operands into the tile's column buffer: columns[0, BN) the weight scales (the norm gains for the norm
// epilogue), columns[SECOND, SECOND + BN) up's scales (gated) or the bias as floats, columns[2 BN, 3 BN) the q/k norm's
// gains; the linears have no scales and the mix and residual epilogues no second operand, so theirs share the one array
// (SECOND = 0).
template <int EPI, int BN, int SECOND>
FRY_DEVICE void store_columns(float* columns, const ColumnLoad& c, int i) {
    if constexpr (scaled(EPI)) columns[i] = c.scale;
    if constexpr (EPI == kEpiLinearNorm) columns[i] = h2f_bits(c.gain);
    if constexpr (EPI == kEpiGated || EPI == kEpiLinearF32) columns[SECOND + i] = c.second;
    if constexpr (biased(EPI) || linear16(EPI) || EPI == kEpiGatedF16) columns[SECOND + i] = h2f_bits(c.half);
    if constexpr (EPI == kEpiBiasQkNorm) columns[2 * BN + i] = h2f_bits(c.gain);
}

// Issues the TMA loads of one sub-tile's row operands (the boxes of its columns below N, none past it) into a slot,
// completing on bar.
template <int EPI, int SUB>
FRY_DEVICE void load_sub_rows(const CUtensorMap* map_residual, const CUtensorMap* map_original, uint8_t* slot, uint64_t* bar, int m0,
                              int n0, int N) {
    constexpr int kBoxes = SUB / kBoxCols, kTensors = mixes(EPI) ? 2 : 1;
    const int in_range = n0 < N ? (N - n0 + kBoxCols - 1) / kBoxCols : 0;
    const int boxes = in_range < kBoxes ? in_range : kBoxes;
    mbar_arrive_expect_tx(bar, boxes * kTensors * kBoxBytes);
    for (int b = 0; b < boxes; ++b) {
        tma_load_2d(slot + b * kBoxBytes, map_residual, bar, n0 + b * kBoxCols, m0);
        if constexpr (mixes(EPI)) tma_load_2d(slot + (kBoxes + b) * kBoxBytes, map_original, bar, n0 + b * kBoxCols, m0);
    }
}

// Where one row's 16-column chunk sits in a staged box: its two 16-byte units (2 (chunk % 4) and the next) of the row's
// 128 bytes, each at its index XOR the row's position in its 8-row swizzle atom.
struct StagedChunk {
    uint8_t* row;  // the row's 128 bytes in the box
    int unit;      // 2 (chunk % 4)
    int swizzle;   // row % 8
    FRY_DEVICE uint4* at(int h) const { return reinterpret_cast<uint4*>(row + (((unit + h) ^ swizzle) << 4)); }
};

// kEpiBiasQkNorm: the attention's q/k RMSNorm on one row's 16 fp16 outputs (as pairs) from output column `column`,
// where they are query or key columns: each head's dq values x (the rounded projection) become fp16((x * inverse) *
// gain), inverse = rsqrt(mean(x^2) + eps). The sums of squares follow the attention kernel's own orders, so the result
// equals what it computes from the unnormalised rows bit for bit: a key's squares in column order; a query's as four
// partial sums (a quad lane's columns 2t, 2t + 1, then 8 + 2t, 9 + 2t) added as (s0 + s1) + (s2 + s3). A head's
// columns lie within the chunk (dq 8 or 16, and the query and key blocks start on 16-column boundaries).
template <int DQ>
FRY_DEVICE void normalize_qk_heads(const GemmArgs& p, bool key, const float* gains, uint32_t (&result)[8]) {
    float gain[16], x[16], y[16];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const float4 four = reinterpret_cast<const float4*>(gains)[q];
        gain[4 * q] = four.x, gain[4 * q + 1] = four.y, gain[4 * q + 2] = four.z, gain[4 * q + 3] = four.w;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        x[2 * i] = h2f_exact(static_cast<uint16_t>(result[i] & 0xffff));
        x[2 * i + 1] = h2f_exact(static_cast<uint16_t>(result[i] >> 16));
    }
    constexpr float kReciprocal = 1.0f / DQ;  // exact: the mean as the attention takes it
#pragma unroll
    for (int first = 0; first < 16; first += DQ) {
        float squares = 0.0f;
        if (key) {
#pragma unroll
            for (int i = 0; i < DQ; ++i) squares = __fmaf_rn(x[first + i], x[first + i], squares);
        } else {
            float s[4];
#pragma unroll
            for (int lane = 0; lane < 4; ++lane) {
                s[lane] = __fmaf_rn(x[first + 2 * lane + 1], x[first + 2 * lane + 1], __fmaf_rn(x[first + 2 * lane], x[first + 2 * lane], 0.0f));
                if constexpr (DQ == 16)
                    s[lane] = __fmaf_rn(x[first + 9 + 2 * lane], x[first + 9 + 2 * lane], __fmaf_rn(x[first + 8 + 2 * lane], x[first + 8 + 2 * lane], s[lane]));
            }
            squares = __fadd_rn(__fadd_rn(s[0], s[1]), __fadd_rn(s[2], s[3]));
        }
        const float inverse = rsqrtf(__fadd_rn(__fmul_rn(squares, kReciprocal), p.norm_eps));
#pragma unroll
        for (int i = 0; i < DQ; ++i) y[first + i] = __fmul_rn(__fmul_rn(x[first + i], inverse), gain[first + i]);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) result[i] = pack_half2_rn(y[2 * i], y[2 * i + 1]);
}

// 1 / sqrt(mean(h^2) + eps) of one 24-wide head's fp16 values h, in the attention kernel's order: a key's squares in
// column order; a query's as four partial sums (a quad lane's columns 2t, 2t + 1, 8 + 2t, 9 + 2t, 16 + 2t, 17 + 2t)
// added as (s0 + s1) + (s2 + s3); the mean by division, as the attention takes it for a dq that is not a power of two.
FRY_DEVICE float qk24_inverse(const float (&h)[24], bool key, float eps) {
    float squares = 0.0f;
    if (key) {
#pragma unroll
        for (int i = 0; i < 24; ++i) squares = __fmaf_rn(h[i], h[i], squares);
    } else {
        float s[4];
#pragma unroll
        for (int lane = 0; lane < 4; ++lane) {
            s[lane] = 0.0f;
#pragma unroll
            for (int base = 0; base < 24; base += 8)
                s[lane] = __fmaf_rn(h[base + 2 * lane + 1], h[base + 2 * lane + 1], __fmaf_rn(h[base + 2 * lane], h[base + 2 * lane], s[lane]));
        }
        squares = __fadd_rn(__fadd_rn(s[0], s[1]), __fadd_rn(s[2], s[3]));
    }
    return rsqrtf(__fadd_rn(__fdiv_rn(squares, 24.0f), eps));
}

// kEpiBiasQkNorm at dq 24: a head's 24 columns span this chunk and the one before or after it. The query and key
// blocks start on 48-column boundaries, as do the 192-column tiles, so `phase` (the chunk's column mod 48) places the
// heads: 0, one head of this chunk's 16 and the next chunk's first 8; 16, the end of one (the chunk before's 16, this
// chunk's first 8) and the start of the next (this chunk's last 8, the next chunk's 16); 32, the end of one (the chunk
// before's last 8, this chunk's 16). near[0] and near[1] hold the chunks before and after as fp16 pairs, computed from
// the accumulator as this chunk's are, so every head is normalised from the values the attention would read.
FRY_DEVICE void normalize_qk24(const GemmArgs& p, bool key, int phase, const float* gains, const uint32_t (&near)[2][8], uint32_t (&result)[8]) {
    float x[16], before[16], after[16], h[24], inverse[16];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        x[2 * i] = h2f_exact(static_cast<uint16_t>(result[i] & 0xffff)), x[2 * i + 1] = h2f_exact(static_cast<uint16_t>(result[i] >> 16));
        before[2 * i] = h2f_exact(static_cast<uint16_t>(near[0][i] & 0xffff)), before[2 * i + 1] = h2f_exact(static_cast<uint16_t>(near[0][i] >> 16));
        after[2 * i] = h2f_exact(static_cast<uint16_t>(near[1][i] & 0xffff)), after[2 * i + 1] = h2f_exact(static_cast<uint16_t>(near[1][i] >> 16));
    }
    if (phase == 0) {
#pragma unroll
        for (int i = 0; i < 24; ++i) h[i] = i < 16 ? x[i] : after[i - 16];
        const float one = qk24_inverse(h, key, p.norm_eps);
#pragma unroll
        for (int i = 0; i < 16; ++i) inverse[i] = one;
    } else if (phase == 16) {
#pragma unroll
        for (int i = 0; i < 24; ++i) h[i] = i < 16 ? before[i] : x[i - 16];
        const float first = qk24_inverse(h, key, p.norm_eps);
#pragma unroll
        for (int i = 0; i < 24; ++i) h[i] = i < 8 ? x[8 + i] : after[i - 8];
        const float second = qk24_inverse(h, key, p.norm_eps);
#pragma unroll
        for (int i = 0; i < 16; ++i) inverse[i] = i < 8 ? first : second;
    } else {
#pragma unroll
        for (int i = 0; i < 24; ++i) h[i] = i < 8 ? before[8 + i] : x[i - 8];
        const float one = qk24_inverse(h, key, p.norm_eps);
#pragma unroll
        for (int i = 0; i < 16; ++i) inverse[i] = one;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i)
        result[i] = pack_half2_rn(__fmul_rn(__fmul_rn(x[2 * i], inverse[2 * i]), gains[2 * i]),
                                  __fmul_rn(__fmul_rn(x[2 * i + 1], inverse[2 * i + 1]), gains[2 * i + 1]));
}

// The bias epilogue's fp16 outputs of one row's 16 columns as pairs, by epilogue16's arithmetic for them: the q/k norm
// at dq 24 reads a head's columns in the chunks beside its own.
FRY_DEVICE void biased_pairs(float xs, const uint32_t (&acc)[16], const float* scale, const float* second, uint32_t (&pairs)[8]) {
    const uint64_t xs2 = pair2(xs, xs);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const float4 a = reinterpret_cast<const float4*>(scale)[q];
        const float4 b = reinterpret_cast<const float4*>(second)[q];
        const float2 low = lanes(fma2(mul2(pair2(static_cast<float>(static_cast<int32_t>(acc[4 * q])), static_cast<float>(static_cast<int32_t>(acc[4 * q + 1]))), xs2),
                                      pair2(a.x, a.y), pair2(b.x, b.y)));
        const float2 high = lanes(fma2(mul2(pair2(static_cast<float>(static_cast<int32_t>(acc[4 * q + 2])), static_cast<float>(static_cast<int32_t>(acc[4 * q + 3]))), xs2),
                                       pair2(a.z, a.w), pair2(b.z, b.w)));
        pairs[2 * q] = pack_half2_rn(low.x, low.y);
        pairs[2 * q + 1] = pack_half2_rn(high.x, high.y);
    }
}

// gains: the chunk's 16 column gains in shared memory (staged with the tile's column operands); near: at dq 24, the
// chunks before and after (normalize_qk24)
FRY_DEVICE void normalize_qk(const GemmArgs& p, int column, const float* gains, const uint32_t (&near)[2][8], uint32_t (&result)[8]) {
    if (column >= p.qk_keys) return;
    const bool key = column >= p.qk_queries;
    if (p.qk_dq == 8) normalize_qk_heads<8>(p, key, gains, result);
    else if (p.qk_dq == 16) normalize_qk_heads<16>(p, key, gains, result);
    else normalize_qk24(p, key, column % 48, gains, near, result);
}

// Applies the epilogue to one row's 16 consecutive columns. acc (and up, gated) hold the raw TMEM words, xs the row's
// activation scale, rs and is the next block's input-mix scales, scale and second the chunk's column operands in shared
// memory. Staged epilogues read the row's residual (and original) from its staged chunk and write the fp16 results over
// it (and into result, as fp16 pairs); int32 and fp32 epilogues store [n, n + valid) of row index `row` directly.
// gains and near: the q/k norm's column gains and, at dq 24, the fp16 outputs of the chunks beside this one.
template <int EPI>
FRY_DEVICE void epilogue16(const GemmArgs& p, float xs, float rs, float is, const uint32_t (&acc)[16], const uint32_t (&up)[16],
                           const float* scale, const float* second, const StagedChunk& staged, const StagedChunk& original, size_t row,
                           int valid, int column, const float* gains, const uint32_t (&near)[2][8], uint32_t (&result)[8]) {
    if constexpr (EPI == kEpiInt32) {
        int32_t* out = static_cast<int32_t*>(p.out) + row;
#pragma unroll
        for (int v = 0; v < 4; ++v)
            if (v * 4 < valid)
                reinterpret_cast<int4*>(out)[v] = make_int4(acc[4 * v], acc[4 * v + 1], acc[4 * v + 2], acc[4 * v + 3]);
        return;
    } else if constexpr (EPI == kEpiLinearF32) {
        float* out = static_cast<float*>(p.out) + row;
#pragma unroll
        for (int q = 0; q < 4; ++q)
            if (q * 4 < valid) {
                const float4 b = reinterpret_cast<const float4*>(second)[q];
                reinterpret_cast<float4*>(out)[q] =
                    make_float4(__fadd_rn(__uint_as_float(acc[4 * q]), b.x), __fadd_rn(__uint_as_float(acc[4 * q + 1]), b.y),
                                __fadd_rn(__uint_as_float(acc[4 * q + 2]), b.z), __fadd_rn(__uint_as_float(acc[4 * q + 3]), b.w));
            }
        return;
    } else {
        constexpr bool kResidual = EPI == kEpiResidual || mixes(EPI) || linear16(EPI);
        uint4 residual_words[2] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)}, original_words[2] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)};
        if constexpr (kResidual) {
            if (!linear16(EPI) || p.residual != nullptr) residual_words[0] = *staged.at(0), residual_words[1] = *staged.at(1);
        }
        if constexpr (mixes(EPI)) original_words[0] = *original.at(0), original_words[1] = *original.at(1);
        const uint16_t* res = reinterpret_cast<const uint16_t*>(residual_words);
        const uint16_t* orig = reinterpret_cast<const uint16_t*>(original_words);
        // the chunk's column operands as 4 x float4 each (the chunk starts on a 64-byte boundary of the staged columns)
        float scale_v[16], second_v[16];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            if constexpr (scaled(EPI)) {
                const float4 a = reinterpret_cast<const float4*>(scale)[q];
                scale_v[4 * q] = a.x, scale_v[4 * q + 1] = a.y, scale_v[4 * q + 2] = a.z, scale_v[4 * q + 3] = a.w;
            }
            if constexpr (biased(EPI) || EPI == kEpiGated || linear16(EPI) || EPI == kEpiGatedF16) {
                const float4 b = reinterpret_cast<const float4*>(second)[q];
                second_v[4 * q] = b.x, second_v[4 * q + 1] = b.y, second_v[4 * q + 2] = b.z, second_v[4 * q + 3] = b.w;
            }
        }
        // the arithmetic two columns at a time in paired fp32 (f32x2: each lane rounds as the scalar instruction does); fp16
        // operands widen on the FMA pipe (h2f_exact)
        const uint64_t xs2 = pair2(xs, xs);
        float values[16];
#pragma unroll
        for (int e = 0; e < 16; e += 2) {
            const uint64_t scale2 = pair2(scale_v[e], scale_v[e + 1]), second2 = pair2(second_v[e], second_v[e + 1]);
            // int8: the int32 sums; fp16: the fp32 sums
            const uint64_t acc2 = scaled(EPI)
                                      ? pair2(static_cast<float>(static_cast<int32_t>(acc[e])), static_cast<float>(static_cast<int32_t>(acc[e + 1])))
                                      : pair2(__uint_as_float(acc[e]), __uint_as_float(acc[e + 1]));
            uint64_t value2;
            if constexpr (biased(EPI)) {
                value2 = fma2(mul2(acc2, xs2), scale2, second2);
            } else if constexpr (EPI == kEpiScaleBf16) {
                value2 = mul2(mul2(acc2, xs2), scale2);
            } else if constexpr (EPI == kEpiGated || EPI == kEpiGatedF16) {
                uint64_t gate2, up2;
                if constexpr (EPI == kEpiGated) {
                    gate2 = mul2(mul2(acc2, xs2), scale2);
                    up2 = mul2(mul2(pair2(static_cast<float>(static_cast<int32_t>(up[e])), static_cast<float>(static_cast<int32_t>(up[e + 1]))), xs2),
                               second2);
                } else {  // the bias (zero when there is none) on the gate alone
                    gate2 = add2(acc2, second2);
                    up2 = pair2(__uint_as_float(up[e]), __uint_as_float(up[e + 1]));
                }
                // silu(g) = g * sigmoid(g), sigmoid from the 2^x and reciprocal instructions: 1 / (1 + 2^(-g log2 e)), the
                // denominator from 1 to infinity
                const float2 power = lanes(mul2(gate2, pair2(-1.4426950408889634f, -1.4426950408889634f)));
                const float2 denominator = lanes(add2(pair2(ex2_approx_ftz(power.x), ex2_approx_ftz(power.y)), pair2(1.0f, 1.0f)));
                const uint64_t sigmoid2 = pair2(rcp_approx_ftz(denominator.x), rcp_approx_ftz(denominator.y));
                value2 = mul2(mul2(gate2, sigmoid2), up2);
            } else if constexpr (EPI == kEpiResidual || EPI == kEpiMix) {
                value2 = fma2(mul2(acc2, xs2), scale2, pair2(h2f_exact(res[e]), h2f_exact(res[e + 1])));
            } else {  // the fp16 linears: (acc + bias) + residual
                value2 = add2(acc2, second2);
                if (p.residual) value2 = add2(value2, pair2(h2f_exact(res[e]), h2f_exact(res[e + 1])));
            }
            if constexpr (mixes(EPI)) {
                // the residual sum rounded to fp16, then mixed with the original
                const float2 sum = lanes(value2);
                const uint32_t stream = pack_half2_rn(sum.x, sum.y);
                const uint64_t stream2 = pair2(h2f_exact(static_cast<uint16_t>(stream & 0xffff)), h2f_exact(static_cast<uint16_t>(stream >> 16)));
                value2 = fma2(stream2, pair2(rs, rs), mul2(pair2(h2f_exact(orig[e]), h2f_exact(orig[e + 1])), pair2(is, is)));
            }
            const float2 value = lanes(value2);
            values[e] = value.x;
            values[e + 1] = value.y;
        }
        // two fp16 (bf16) roundings an instruction, over the staged residual
#pragma unroll
        for (int i = 0; i < 8; ++i)
            result[i] = EPI == kEpiScaleBf16 ? pack_bf162_rn(values[2 * i], values[2 * i + 1]) : pack_half2_rn(values[2 * i], values[2 * i + 1]);
        if constexpr (EPI == kEpiBiasQkNorm) normalize_qk(p, column, gains, near, result);
        *staged.at(0) = make_uint4(result[0], result[1], result[2], result[3]);
        *staged.at(1) = make_uint4(result[4], result[5], result[6], result[7]);
    }
}

// The prologue of a normed A: the epilogue warps (warp w: rows w, w + 16, ... of the block) turn the block's fp16 rows of
// p.norm_x into int8 rows of the resident A, zero past M, and their scales into row_scales.
template <int NKS>
FRY_DEVICE void norm_rows_into_a(const GemmArgs& p, uint8_t* resident, float* row_scales, int m0, int M, int warp, int lane) {
    constexpr int kChunks = NKS / 2, K = NKS * kTileKBytes;      // 256 columns a chunk, 128 a slice
    constexpr int kRows = kBlockM / kEpilogueWarps, kAhead = 2;  // rows of a warp; rows in flight beyond the one worked on
    float gain[kChunks][8];
    load_gain<kChunks>(p.norm_gain, K, lane, gain);
    const uint64_t unused = pair2(0.0f, 0.0f);
    const uint4 no_original[1] = {make_uint4(0, 0, 0, 0)};
    uint4 raw[kRows][kChunks];  // unrolled: kAhead + 1 of them live at a time
    auto load = [&](int i) {
        const int row = m0 + warp + i * kEpilogueWarps;
        if (row < M) {
            load_row_chunks<kChunks>(p.norm_x + static_cast<size_t>(row) * K, K, lane, raw[i]);
        } else {
#pragma unroll
            for (int c = 0; c < kChunks; ++c) raw[i][c] = make_uint4(0, 0, 0, 0);
        }
    };
#pragma unroll
    for (int i = 0; i < kAhead; ++i) load(i);
#pragma unroll
    for (int i = 0; i < kRows; ++i) {
        if (i + kAhead < kRows) load(i + kAhead);
        const int r = warp + i * kEpilogueWarps;
        const SwizzledRowOut out{resident, r};
        if (m0 + r < M) {  // uniform across the warp
            norm_quant_row<kChunks, false, SwizzledRowOut>(raw[i], no_original, gain, unused, unused, p.norm_eps, K, lane, nullptr, out,
                                                           row_scales + r);
        } else {  // a row past M: zeros, so its accumulator rows stay 0
#pragma unroll
            for (int c = 0; c < kChunks; ++c)
                if ((c * 32 + lane) * 8 < K) out.put8((c * 32 + lane) * 8, make_uint2(0u, 0u));
            if (lane == 0) row_scales[r] = 0.0f;
        }
    }
}

FRY_DEVICE void norm_sync() { asm volatile("bar.sync %0, %1;" ::"n"(kNormBarrier), "n"(kEpilogueThreads) : "memory"); }

// kEpiLinearNorm, after a tile's epilogue: norm_quant of the tile's 128 rows, whose 768 (or N) columns lie in the N / BN
// CTAs of this cluster, one column tile each. Each thread holds its row's fp16 outputs of its chunks (kept) and their
// partial sum of squares and largest |x * gain|. The 4 threads of a row add theirs in shared memory; each rank's row
// partials go to every rank (distributed shared memory, an arrival on each rank's xready); each thread then adds the
// ranks' partials in rank order, and quantises its kept values: inverse = 1 / sqrt(sum / N + eps), absmax = inverse *
// the largest |x * gain| (the largest |(x * inverse) * gain| to within fp32 rounding), q = rint((x * inverse) * gain *
// 127 / absmax), the row's scale absmax / 127 (written by rank 0). A thread whose earlier wait timed out still takes every
// barrier and arrival, so no rank waits on it for ever.
template <typename S, int KEPT>
FRY_DEVICE void norm_rows_of_tile(const GemmArgs& p, float* norm_smem, uint64_t* xready, const float* columns, const uint32_t (&kept)[KEPT][8],
                                  float squares, float largest, int local, int m, int n0, int M, int N, int ranks, int row, int part,
                                  int lane, bool& alive) {
    const int tb = local & 1;  // exchange buffer and barrier of this tile (tiles alternate)
    float* exchange = norm_smem;                              // [2][kMaxCluster][128][2]
    float* parts = norm_smem + 2 * kMaxCluster * kBlockM * 2;  // [2][4][128]
    parts[part * kBlockM + row] = squares;
    parts[(kChunkParts + part) * kBlockM + row] = largest;
    norm_sync();
    const uint32_t rank = cluster_rank();
    if (part == 0) {  // warps 0-3: a thread a row
        float sum = parts[row], top = parts[kChunkParts * kBlockM + row];
#pragma unroll
        for (int q = 1; q < kChunkParts; ++q) {
            sum = __fadd_rn(sum, parts[q * kBlockM + row]);
            top = fmaxf(top, parts[(kChunkParts + q) * kBlockM + row]);
        }
        float* mine = exchange + ((tb * kMaxCluster + rank) * kBlockM + row) * 2;
        for (int peer = 0; peer < ranks; ++peer) st_peer_f32x2(peer_smem(mine, peer), sum, top);
        __syncwarp();
        if (lane == 0)
            for (int peer = 0; peer < ranks; ++peer) mbar_arrive_peer(peer_smem(&xready[tb], peer));
    }
    if (!mbar_wait_cluster(&xready[tb], (local >> 1) & 1, 17)) alive = false;
    if (!alive) return;
    float sum = 0.0f, top = 0.0f;
    for (int r = 0; r < ranks; ++r) {
        const float* entry = exchange + ((tb * kMaxCluster + r) * kBlockM + row) * 2;
        sum = r == 0 ? entry[0] : __fadd_rn(sum, entry[0]);
        top = fmaxf(top, entry[1]);
    }
    const float inverse = rsqrtf(__fadd_rn(__fdiv_rn(sum, static_cast<float>(N)), p.norm_eps));
    const float absmax = fmaxf(__fmul_rn(inverse, top), 1e-20f);
    const float step_inverse = __fdiv_rn(127.0f, absmax);
    if (m >= M) return;
    if (rank == 0 && part == 0) p.norm_scale[m] = __fdiv_rn(absmax, 127.0f);
    const uint64_t inverse2 = pair2(inverse, inverse);
#pragma unroll
    for (int k = 0; k < KEPT; ++k) {
        const int sub = k / S::kChunksPerSub, c = sub * S::kSub + part * kChunkCols + (k % S::kChunksPerSub) * kChunkCols * kChunkParts;
        uint2 bytes[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            float y[8];
#pragma unroll
            for (int i = 0; i < 8; i += 2) {
                const uint32_t pair = kept[k][h * 4 + i / 2];
                const float2 v = lanes(mul2(mul2(pair2(h2f_exact(static_cast<uint16_t>(pair & 0xffff)), h2f_exact(static_cast<uint16_t>(pair >> 16))),
                                                 inverse2),
                                            pair2(columns[c + h * 8 + i], columns[c + h * 8 + i + 1])));
                y[i] = v.x;
                y[i + 1] = v.y;
            }
            bytes[h] = quantize8(y, step_inverse);
        }
        *reinterpret_cast<uint4*>(p.norm_q + static_cast<size_t>(m) * N + n0 + c) = make_uint4(bytes[0].x, bytes[0].y, bytes[1].x, bytes[1].y);
    }
}

template <int KIND, int BN, bool GATED, int EPI, int SUB, int NKS, bool PAIR>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                const __grid_constant__ CUtensorMap map_out, const __grid_constant__ CUtensorMap map_residual,
                const __grid_constant__ CUtensorMap map_original, const GemmArgs args, int M, int N, int K) {
    using S = GemmShape<KIND, BN, GATED, EPI, SUB, NKS, PAIR>;
    extern __shared__ __align__(1024) uint8_t smem[];
    if (smem_addr(smem) & 1023u) {  // uniform across the CTA: every thread leaves before any barrier
        if (threadIdx.x == 0) record_error(kMisaligned, 20);
        if constexpr (EPI == kEpiLinearNorm || PAIR) cluster_sync();  // its peers leave the same way
        return;
    }
    uint8_t* resident = smem;                                            // a normed A: [NKS][128 rows][128 bytes, swizzled]
    uint8_t* stages = smem + S::kResidentBytes;                          // [kStages][A box | B box(es)]
    uint8_t* io = stages + S::kStages * S::kStageBytes;                  // [kSlots][tensors][kBoxes][128 rows][128 bytes, swizzled]
    float* column_buffers = reinterpret_cast<float*>(io + S::kIoBytes);  // [2][2 * BN]
    float* row_scales = reinterpret_cast<float*>(io + S::kIoBytes + S::kColumnBytes);  // a normed A's [128]
    float* norm_smem = reinterpret_cast<float*>(io + S::kIoBytes + S::kColumnBytes + S::kRowScaleBytes);  // kEpiLinearNorm's
    uint64_t* full = reinterpret_cast<uint64_t*>(io + S::kIoBytes + S::kColumnBytes + S::kRowScaleBytes + S::kNormBytes);
    uint64_t* empty = full + S::kStages;
    uint64_t* tmem_full = empty + S::kStages;   // [2]: an accumulator is ready for the epilogue
    uint64_t* tmem_empty = tmem_full + 2;       // [2]: the epilogue has read an accumulator out
    uint64_t* rows_full = tmem_empty + 2;       // [kSlots]: a slot's row operands have landed
    uint64_t* a_ready = rows_full + 3;          // a normed A's block is in place (all epilogue warps)
    uint64_t* xready = a_ready + 1;             // [2]: every rank's row partials of a tile have arrived (kEpiLinearNorm)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(xready + 2);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_blocks = (N + BN - 1) / BN;
    // PAIR: a tile is the pair's 256 rows, of which this CTA (cluster rank 0 or 1) takes 128 from 128 * rank; the
    // pairs walk the tiles as single CTAs do
    constexpr int kTileRows = PAIR ? 2 * kBlockM : kBlockM;
    const int rank = PAIR ? static_cast<int>(cluster_rank()) : 0;
    const int workers = PAIR ? static_cast<int>(gridDim.x) / 2 : static_cast<int>(gridDim.x);
    const int worker = PAIR ? static_cast<int>(blockIdx.x) / 2 : static_cast<int>(blockIdx.x);
    const int row_blocks = (M + kTileRows - 1) / kTileRows;
    const int tiles = row_blocks * n_blocks;
    auto row0 = [&](int tile) { return (tile / n_blocks) * kTileRows + rank * kBlockM; };  // this CTA's first row
    const int k_tiles = (K * S::kElem + kTileKBytes - 1) / kTileKBytes;
    // Tile order (tile = row block * n_blocks + column tile). Plain: round robin over the tiles. Normed A: round robin over
    // units, a unit being a row block's column tiles g, g + groups, ... (groups = gridDim.x / row_blocks, at least 1, the
    // launch's choice), so a CTA makes a unit's A once and reuses it for each of the unit's tiles.
    const int groups = NKS > 0 ? max(1, static_cast<int>(gridDim.x) / row_blocks) : 1;
    auto unit_tile = [&](int unit) { return (unit / groups) * n_blocks + unit % groups; };
    const int first_tile = NKS > 0 ? unit_tile(blockIdx.x) : worker;
    auto next_tile = [&](int tile) {
        if (NKS == 0) return tile + workers;
        const int column = tile % n_blocks;
        if (column + groups < n_blocks) return tile + groups;
        const int unit = (tile / n_blocks) * groups + column % groups + static_cast<int>(gridDim.x);
        return unit / groups < row_blocks ? unit_tile(unit) : tiles;
    };
    auto unit_start = [&](int tile) { return NKS > 0 && tile % n_blocks < groups; };
    // a tile's first output column. Normed A: row block b takes its column tiles rotated by b, so the CTAs, which start
    // their units together, stream different B tiles rather than all the same one
    auto column0 = [&](int tile) {
        const int column = tile % n_blocks;
        return (NKS > 0 ? (column + tile / n_blocks) % n_blocks : column) * BN;
    };
    // sub-tiles in the order this CTA takes them: (tile, s) -> (tile, s + 1), or the next tile's first
    auto advance = [&](int& tile, int& sub) {
        if (++sub == S::kSubs) {
            sub = 0;
            tile = next_tile(tile);
        }
    };

    if (threadIdx.x == 0) {
        for (int s = 0; s < S::kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tmem_full[b], 1);
            mbar_init(&tmem_empty[b], PAIR ? 2 * kEpilogueWarps : kEpilogueWarps);  // PAIR: both CTAs' warps, on the even CTA's
        }
        for (int b = 0; b < S::kSlots; ++b) mbar_init(&rows_full[b], 1);
        mbar_init(a_ready, kEpilogueWarps);
        for (int b = 0; b < 2; ++b) mbar_init(&xready[b], EPI == kEpiLinearNorm ? n_blocks * 4 : 1);  // 4 warps a rank
        fence_barrier_init();
    }
    if (warp == 0) {
        if constexpr (PAIR) {
            tmem_alloc_pair(tmem_slot, S::kTmemCols);
            tmem_relinquish_pair();
        } else {
            tmem_alloc(tmem_slot, S::kTmemCols);
            tmem_relinquish();
        }
    }
    if (warp == kProducerWarp && lane == 0) {
        prefetch_tensor_map(&map_a);
        prefetch_tensor_map(&map_b);
    }
    tc_fence_before();
    __syncthreads();
    if constexpr (EPI == kEpiLinearNorm || PAIR) cluster_sync();  // every rank's barriers are initialised before any remote arrival
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // weights that no earlier kernel writes (args.b_constant): the producer loads B of the first stages (the ring is
    // empty) before waiting for the earlier kernels, so those loads overlap their tail; A follows after the wait, into
    // the same stages, whose barriers expect both
    // A stage's loads. PAIR: both CTAs' loads (each its A rows and its half of B) complete on the even CTA's stage
    // barrier, which its producer arms for the pair's bytes; the odd CTA's producer does not arrive
    auto arm_stage = [&](int s) {
        if (!PAIR || rank == 0) mbar_arrive_expect_tx(&full[s], (PAIR ? 2 : 1) * S::kStageBytes);
    };
    auto load_b = [&](uint8_t* b, int s, int kt, int n0) {
        if constexpr (PAIR) {
            const int rows = GATED ? (rank == 0 ? n0 : N + n0) : n0 + rank * S::kBRows;
            tma_load_2d_pair(b, &map_b, peer_smem(&full[s], 0), kt * S::kBoxK, rows);
        } else {
            tma_load_2d(b, &map_b, &full[s], kt * S::kBoxK, n0);
            if constexpr (GATED) tma_load_2d(b + S::kBBytes, &map_b, &full[s], kt * S::kBoxK, N + n0);
        }
    };
    auto load_a = [&](uint8_t* a, int s, int kt, int m0) {
        if constexpr (PAIR) tma_load_2d_pair(a, &map_a, peer_smem(&full[s], 0), kt * S::kBoxK, m0);
        else tma_load_2d(a, &map_a, &full[s], kt * S::kBoxK, m0);
    };
    int preloaded = 0;
    if (args.b_constant && warp == kProducerWarp && elect_one()) {
        for (int tile = first_tile, kt = 0; preloaded < S::kStages && tile < tiles; ++preloaded) {
            uint8_t* b = stages + preloaded * S::kStageBytes + (NKS > 0 ? 0 : S::kABytes);
            arm_stage(preloaded);
            load_b(b, preloaded, kt, column0(tile));
            if (++kt == k_tiles) {
                kt = 0;
                tile = next_tile(tile);
            }
        }
    }
    grid_dependency_start();  // setup done: now the operands of earlier kernels

    if (warp == kProducerWarp) {
        if (elect_one()) {
            int it = 0;
            bool ok = true;
            for (int tile = first_tile; tile < tiles && ok; tile = next_tile(tile)) {
                const int m0 = row0(tile), n0 = column0(tile);
                for (int kt = 0; kt < k_tiles; ++kt, ++it) {
                    const int s = it % S::kStages;
                    const uint32_t phase = (it / S::kStages) & 1;
                    uint8_t* a = stages + s * S::kStageBytes;
                    uint8_t* b = NKS > 0 ? a : a + S::kABytes;
                    if (it >= preloaded) {  // a preloaded stage has its barrier armed and its B in flight
                        // PAIR: the even CTA's MMA warp frees the stage in both CTAs (its commit arrives on both)
                        if (!mbar_wait(&empty[s], phase ^ 1, 10)) {
                            ok = false;
                            break;
                        }
                        arm_stage(s);
                        load_b(b, s, kt, n0);
                    }
                    if constexpr (NKS == 0) load_a(a, s, kt, m0);
                }
            }
        }
    } else if (warp == kMmaWarp) {
        // PAIR: the even CTA issues the pair's MMAs and frees stages and hands over accumulators in both CTAs
        auto commit = [&](uint64_t* bar) {
            if constexpr (PAIR) {
                mma_commit_pair(smem_addr(bar));
                mma_commit_pair(peer_smem(bar, 1));
            } else {
                mma_commit(bar);
            }
        };
        if ((!PAIR || rank == 0) && elect_one()) {
            // gated: the gate's and the up's B boxes lie back to back, 2 BN rows at the swizzle's 1024 bytes per 8, so one MMA of
            // N = 2 BN fills both accumulator halves
            constexpr uint32_t idesc = instr_desc<KIND>(S::kAccCols, kTileRows);
            int it = 0, local = 0, units = 0;
            bool ok = true;
            for (int tile = first_tile; tile < tiles && ok; tile = next_tile(tile), ++local) {
                const int buffer = local & 1;
                if (unit_start(tile) && !mbar_wait(a_ready, (units++) & 1, 16)) break;  // the unit's A is made
                if (!mbar_wait(&tmem_empty[buffer], ((local >> 1) & 1) ^ 1, 11)) break;
                tc_fence_after();
                const uint32_t accumulator = tmem + buffer * S::kAccCols;
                for (int kt = 0; kt < k_tiles; ++kt, ++it) {
                    const int s = it % S::kStages;
                    const uint32_t phase = (it / S::kStages) & 1;
                    if (!mbar_wait(&full[s], phase, 12)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t stage = smem_addr(stages + s * S::kStageBytes);
                    const uint32_t a = NKS > 0 ? smem_addr(resident) + kt * S::kABytes : stage;
                    const uint32_t b = NKS > 0 ? stage : stage + S::kABytes;
#pragma unroll
                    for (int k = 0; k < kTileKBytes / kMmaKBytes; ++k) {
                        const uint64_t da = smem_desc_sw128(a + k * kMmaKBytes);
                        const uint32_t accumulate = (kt > 0 || k > 0) ? 1u : 0u;
                        if constexpr (PAIR) mma_ss_pair<KIND>(accumulator, da, smem_desc_sw128(b + k * kMmaKBytes), idesc, accumulate);
                        else mma_ss<KIND>(accumulator, da, smem_desc_sw128(b + k * kMmaKBytes), idesc, accumulate);
                    }
                    commit(&empty[s]);
                }
                commit(&tmem_full[buffer]);
            }
        }
    } else if (warp == kStoreWarp) {
        // the staged sub-tiles' TMA traffic: after sub-tile j's barrier, its stores from slot j % kSlots; once they have
        // read the slot, the row operands of sub-tile j + kSlots into it (those of the first kSlots sub-tiles first).
        // Sub-tile j + kSlots is staged into the slot after barrier j + kSlots - 1, which this warp reaches only once the
        // reads are done: with row operands it waits for them here, before loading the rows; without, it waits for all
        // but the last kSlots - 2 groups, so sub-tile j's stores keep reading while the next kSlots - 2 sub-tiles stage.
        if constexpr (S::kStaged) {
            const bool has_rows = S::kRowTensors > 0 && (!linear16(EPI) || args.residual != nullptr);
            const bool issuer = lane == 0;
            auto load_rows = [&](int tile, int sub, int slot) {
                if (!issuer || !has_rows || tile >= tiles) return;
                load_sub_rows<EPI, SUB>(&map_residual, &map_original, io + slot * S::kSlotBytes, &rows_full[slot],
                                        row0(tile), column0(tile) + sub * SUB, N);
            };
            int ahead_tile = first_tile, ahead_sub = 0;  // the sub-tile kSlots ahead of the one being stored
            for (int slot = 0; slot < S::kSlots; ++slot) {
                load_rows(ahead_tile, ahead_sub, slot);
                advance(ahead_tile, ahead_sub);
            }
            epilogue_sync();  // the first tile's column operands are staged
            int j = 0;
            for (int tile = first_tile; tile < tiles; tile = next_tile(tile)) {
                for (int sub = 0; sub < S::kSubs; ++sub, ++j) {
                    const int slot = j % S::kSlots;
                    __syncwarp();
                    epilogue_sync();  // sub-tile j is staged
                    if (issuer) {
                        const int m0 = row0(tile), n0 = column0(tile) + sub * SUB;
                        uint8_t* staged = io + slot * S::kSlotBytes;
                        for (int b = 0; b < S::kBoxes && n0 + b * kBoxCols < N; ++b)
                            tma_store_2d(&map_out, staged + b * kBoxBytes, n0 + b * kBoxCols, m0);
                        bulk_commit();
                        if (has_rows) bulk_wait_read_all();
                        else bulk_wait_read<S::kSlots - 2>();
                    }
                    load_rows(ahead_tile, ahead_sub, slot);
                    advance(ahead_tile, ahead_sub);
                }
            }
            if (issuer) bulk_wait_all();
        } else {
            epilogue_sync();
            for (int tile = first_tile; tile < tiles; tile = next_tile(tile)) epilogue_sync();
        }
    } else {
        // warps 0-15: warp w reads TMEM lanes 32 (w % 4) .. +31 (rows m0 + 32 (w % 4) + lane) and the 16-column chunks
        // w / 4, w / 4 + 4, ...
        const int quarter = warp & 3, part = warp >> 2;
        const int row_in_tile = quarter * 32 + lane;
        float rs = 0.0f, is = 0.0f;
        if constexpr (mixes(EPI)) {
            rs = h2f_bits(*args.residual_scale);
            is = h2f_bits(*args.input_scale);
        }
        const bool has_rows = S::kRowTensors > 0 && (!linear16(EPI) || args.residual != nullptr);
        auto tile_origin = [&](int tile, int& m0, int& n0) {
            m0 = row0(tile);
            n0 = column0(tile);
        };
        // a tile's column operands (thread i < BN: column n0 + i) and this thread's row scale are loaded into registers
        // at the start of the tile before (the first tile's here) and the column operands written at its end into the
        // other of two column buffers, so one barrier a tile publishes both the staged outputs and them
        static_assert(BN <= kEpilogueThreads, "an epilogue thread stages at most one column");
        bool alive = true;
        float xs_next = 0.0f;
        ColumnLoad column_next;
        auto load_operands = [&](int tile) {
            int m0, n0;
            tile_origin(tile, m0, n0);
            const int m = m0 + row_in_tile;
            if constexpr (scaled(EPI) && NKS == 0) xs_next = (alive && m < M) ? args.x_scale[m] : 0.0f;
            if constexpr (EPI != kEpiInt32)
                if (threadIdx.x < BN) column_next = load_columns<EPI>(args, n0 + static_cast<int>(threadIdx.x), N);
        };
        auto store_operands = [&](int buffer) {
            if constexpr (EPI != kEpiInt32)
                if (threadIdx.x < BN) store_columns<EPI, BN, S::kSecond>(column_buffers + buffer * S::kColumnArrays * BN, column_next, threadIdx.x);
        };
        load_operands(first_tile);
        store_operands(0);
        epilogue_sync();
        // a warp whose wait timed out keeps walking the tiles (and the named barrier) without touching them, so the other
        // epilogue warps never wait at the barrier for it
        int local = 0, j = 0, units = 0;
        float xs_unit = 0.0f;
        for (int tile = first_tile; tile < tiles; tile = next_tile(tile), ++local) {
            const int buffer = local & 1;
            const int next = next_tile(tile);
            int m0, n0;
            tile_origin(tile, m0, n0);
            const int m = m0 + row_in_tile;
            if constexpr (NKS > 0) {
                if (unit_start(tile)) {
                    // the unit's A: every earlier tile's accumulator has been read, so the MMAs that read the last A are done
                    if (alive) norm_rows_into_a<NKS>(args, resident, row_scales, m0, M, warp, lane);
                    fence_proxy_async_shared();  // this thread's A bytes, visible to the MMAs
                    __syncwarp();
                    if (lane == 0) mbar_arrive(a_ready);
                    if (alive && !mbar_wait(a_ready, (units++) & 1, 15)) alive = false;
                    xs_unit = alive ? row_scales[row_in_tile] : 0.0f;
                }
            }
            const float xs = NKS > 0 ? xs_unit : xs_next;
            if (next < tiles) load_operands(next);  // in flight while this tile is worked on
            if (alive && !mbar_wait(&tmem_full[buffer], (local >> 1) & 1, 13)) alive = false;
            const float* columns = column_buffers + buffer * S::kColumnArrays * BN;
            const uint32_t lane_base = tmem + buffer * S::kAccCols + (static_cast<uint32_t>(quarter * 32) << 16);
            // kEpiLinearNorm: this thread's fp16 outputs (its row, its chunks) and their partial sums for the row's norm:
            // the squares, and the largest |x * gain|
            constexpr int kKept = EPI == kEpiLinearNorm ? S::kSubs * S::kChunksPerSub : 1;
            uint32_t kept[kKept][8];
            float squares = 0.0f, largest = 0.0f;
#pragma unroll(EPI == kEpiLinearNorm ? S::kSubs : 1)
            for (int sub = 0; sub < S::kSubs; ++sub, ++j) {
                // sub-tile j stages into slot j % kSlots, which the stores of sub-tile j - kSlots had read before the barrier that ended
                // sub-tile j - 1; every thread waits for the row operands, alive or not, so none is in flight when the CTA exits
                const int slot = j % S::kSlots;
                if (has_rows && !mbar_wait(&rows_full[slot], (j / S::kSlots) & 1, 14)) alive = false;
                uint8_t* staged_sub = io + slot * S::kSlotBytes;
                if (alive) {
                    tc_fence_after();
#pragma unroll
                    for (int k = 0; k < S::kChunksPerSub; ++k) {
                        const int c = sub * SUB + part * kChunkCols + k * kChunkCols * kChunkParts;
                        if (c >= (sub + 1) * SUB || n0 + c >= N) break;  // uniform
                        // the q/k norm at dq 24: the chunks before and after this one, where its heads reach into them (within
                        // the tile: its columns and the heads' blocks start on 48-column boundaries)
                        uint32_t near[2][8] = {};
                        if constexpr (EPI == kEpiBiasQkNorm && BN % 48 == 0) {
                            if (args.qk_dq == 24 && n0 + c < args.qk_keys) {  // uniform
                                const int phase = (n0 + c) % 48;
                                uint32_t side[16];
                                if (phase != 0) {
                                    tmem_load16(lane_base + c - kChunkCols, side);
                                    tmem_load_wait();
                                    biased_pairs(xs, side, columns + c - kChunkCols, columns + S::kSecond + c - kChunkCols, near[0]);
                                }
                                if (phase != 32) {
                                    tmem_load16(lane_base + c + kChunkCols, side);
                                    tmem_load_wait();
                                    biased_pairs(xs, side, columns + c + kChunkCols, columns + S::kSecond + c + kChunkCols, near[1]);
                                }
                            }
                        }
                        uint32_t acc[16], up[16];
                        tmem_load16(lane_base + c, acc);
                        if constexpr (GATED) tmem_load16(lane_base + BN + c, up);
                        tmem_load_wait();
                        const int c_sub = c - sub * SUB;
                        const int box = c_sub / kBoxCols, unit = 2 * ((c_sub % kBoxCols) / kChunkCols), swizzle = row_in_tile & 7;
                        const StagedChunk staged{staged_sub + box * kBoxBytes + row_in_tile * 128, unit, swizzle};
                        const StagedChunk original{staged_sub + (S::kBoxes + box) * kBoxBytes + row_in_tile * 128, unit, swizzle};
                        const int valid = N - n0 - c >= 16 ? 16 : N - n0 - c;  // 8 or 16: N is a multiple of 8
                        uint32_t result[8];
                        if (S::kStaged || m < M)
                            epilogue16<EPI>(args, xs, rs, is, acc, up, columns + c, columns + S::kSecond + c, staged, original,
                                            static_cast<size_t>(m) * N + n0 + c, valid, n0 + c, columns + 2 * BN + c, near, result);
                        if constexpr (EPI == kEpiLinearNorm) {
#pragma unroll
                            for (int i = 0; i < 8; ++i) {
                                kept[sub * S::kChunksPerSub + k][i] = result[i];
                                const float x0 = h2f_exact(static_cast<uint16_t>(result[i] & 0xffff));
                                const float x1 = h2f_exact(static_cast<uint16_t>(result[i] >> 16));
                                squares = __fmaf_rn(x1, x1, __fmaf_rn(x0, x0, squares));
                                largest = fmaxf(largest, fmaxf(fabsf(__fmul_rn(x0, columns[c + 2 * i])), fabsf(__fmul_rn(x1, columns[c + 2 * i + 1]))));
                            }
                        }
                    }
                }
                if (sub == S::kSubs - 1) {
                    // this warp's reads of the accumulator are complete: the MMA warp may fill it again
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) {
                        if constexpr (PAIR) mbar_arrive_remote(peer_smem(&tmem_empty[buffer], 0));  // the even CTA's MMA warp waits on it
                        else mbar_arrive(&tmem_empty[buffer]);
                    }
                    if (next < tiles) store_operands(buffer ^ 1);
                }
                // this thread's staged writes, visible to the async proxy before the stores read them
                if constexpr (S::kStaged) fence_proxy_async_shared();
                epilogue_sync();
            }
            if constexpr (EPI == kEpiLinearNorm)
                norm_rows_of_tile<S>(args, norm_smem, xready, columns, kept, squares, largest, local, m, n0, M, N, n_blocks, row_in_tile,
                                     part, lane, alive);
        }
    }
    tc_fence_before();
    __syncthreads();
    // PAIR: neither CTA frees the pair's TMEM, or leaves, before the other is done with it and with the even CTA's barriers
    if constexpr (PAIR) cluster_sync();
    if (warp == 0) {
        tc_fence_after();
        if constexpr (PAIR) tmem_dealloc_pair(tmem, S::kTmemCols);
        else tmem_dealloc(tmem, S::kTmemCols);
    }
    // no rank leaves while a peer may still write its shared memory or arrive on its barriers
    if constexpr (EPI == kEpiLinearNorm) cluster_sync();
}

// ---- host side ---------------------------------------------------------------------------------------------

namespace {

using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*, const cuuint64_t*,
                                 const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                 CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encoder(std::string* error) {
    static EncodeTiled fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* symbol = nullptr;
        cudaDriverEntryPointQueryResult found;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &symbol, cudaEnableDefault, &found) == cudaSuccess &&
            found == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiled>(symbol);
    });
    if (!fn && error) *error = "the CUDA driver has no cuTensorMapEncodeTiled";
    return fn;
}

// A [rows, k] K-major operand as a TMA map with a box of 128 bytes of K by box_rows rows, 128-byte swizzle, zero fill.
bool make_map(CUtensorMap* map, const void* base, int elem_bytes, int k, int rows, int box_rows, std::string* error) {
    EncodeTiled encode = encoder(error);
    if (!encode) return false;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(k), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(k) * elem_bytes};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(kTileKBytes / elem_bytes), static_cast<cuuint32_t>(box_rows)};
    const cuuint32_t element_strides[2] = {1, 1};
    const CUresult result = encode(map, elem_bytes == 1 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                                   const_cast<void*>(base), dims, strides, box, element_strides, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (result != CUDA_SUCCESS) {
        if (error) *error = "cuTensorMapEncodeTiled failed with CUresult " + std::to_string(static_cast<int>(result));
        return false;
    }
    return true;
}

// An fp16 (bf16) [rows, cols] row-major tensor as a TMA map with a box of 64 columns by 128 rows in the 128-byte
// swizzle: the boxes the epilogue stages.
bool make_box_map(CUtensorMap* map, const void* base, int cols, int rows, std::string* error, bool bf16 = false) {
    EncodeTiled encode = encoder(error);
    if (!encode) return false;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols) * 2};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(kBoxCols), static_cast<cuuint32_t>(kBlockM)};
    const cuuint32_t element_strides[2] = {1, 1};
    const CUresult result = encode(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base),
                                   dims, strides, box, element_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                   CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (result != CUDA_SUCCESS) {
        if (error) *error = "cuTensorMapEncodeTiled (fp16 [" + std::to_string(rows) + ", " + std::to_string(cols) +
                            "] staging map) failed with CUresult " + std::to_string(static_cast<int>(result));
        return false;
    }
    return true;
}

template <int KIND, int BN, bool GATED, int EPI, int SUB = BN, int NKS = 0, bool PAIR = false>
cudaError_t launch(const void* a, const void* b, const GemmArgs& args, int M, int N, int K, cudaStream_t stream, std::string* error) {
    using S = GemmShape<KIND, BN, GATED, EPI, SUB, NKS, PAIR>;
    auto kernel = gemm_kernel<KIND, BN, GATED, EPI, SUB, NKS, PAIR>;
    const cudaError_t attribute = ensure_smem(reinterpret_cast<const void*>(kernel), S::kSmemBytes);
    if (attribute != cudaSuccess) return attribute;
    CUtensorMap map_a, map_b, map_out, map_residual, map_original;
    if (!make_map(&map_b, b, S::kElem, K, GATED ? 2 * N : N, S::kBRows, error)) return cudaErrorInvalidValue;
    if (NKS > 0) {
        map_a = map_b;  // a normed A is made in shared memory, not loaded
    } else if (!make_map(&map_a, a, S::kElem, K, M, kBlockM, error)) {
        return cudaErrorInvalidValue;
    }
    // the staged epilogues' maps; unused ones repeat the output's, which is always valid
    map_out = map_residual = map_original = map_a;
    if constexpr (S::kStaged) {
        if (!make_box_map(&map_out, args.out, N, M, error, EPI == kEpiScaleBf16)) return cudaErrorInvalidValue;
        map_residual = map_original = map_out;
        if (args.residual && !make_box_map(&map_residual, args.residual, N, M, error)) return cudaErrorInvalidValue;
        if (mixes(EPI) && !make_box_map(&map_original, args.original, N, M, error)) return cudaErrorInvalidValue;
    }
    const int row_blocks = (M + kBlockM - 1) / kBlockM, n_blocks = (N + BN - 1) / BN, tiles = row_blocks * n_blocks;
    int device = 0, multiprocessors = 0;
    cudaError_t status = cudaGetDevice(&device);
    if (status == cudaSuccess) status = cudaDeviceGetAttribute(&multiprocessors, cudaDevAttrMultiProcessorCount, device);
    if (status != cudaSuccess) return status;
    int grid = tiles < multiprocessors ? tiles : multiprocessors;
    if constexpr (PAIR) {
        // CTA pairs, as many as the device holds at once, none without a tile of 256 rows
        const int pair_tiles = ((M + 2 * kBlockM - 1) / (2 * kBlockM)) * n_blocks;
        int clusters = 0;
        status = max_active_clusters(kernel, dim3(kGemmThreads), S::kSmemBytes, 2, &clusters);
        if (status != cudaSuccess) return status;
        if (clusters < 1) {
            if (error) *error = "no CTA pair of this GEMM fits the device";
            return cudaErrorInvalidValue;
        }
        const int pairs = pair_tiles < clusters ? pair_tiles : clusters;
        return launch_dependent_cluster(kernel, dim3(2 * pairs), dim3(kGemmThreads), S::kSmemBytes, 2, stream, map_a, map_b, map_out,
                                        map_residual, map_original, args, M, N, K);
    }
    if constexpr (EPI == kEpiLinearNorm) {
        // clusters of a row block's n_blocks CTAs, as many as the device holds at once (a persistent cluster takes row
        // blocks b, b + clusters, ...)
        int clusters = 0;
        status = max_active_clusters(kernel, dim3(kGemmThreads), S::kSmemBytes, n_blocks, &clusters);
        if (status != cudaSuccess) return status;
        if (clusters < 1) {
            if (error) *error = "no cluster of " + std::to_string(n_blocks) + " GEMM CTAs fits the device";
            return cudaErrorInvalidValue;
        }
        grid = (row_blocks < clusters ? row_blocks : clusters) * n_blocks;
        return launch_dependent_cluster(kernel, dim3(grid), dim3(kGemmThreads), S::kSmemBytes, n_blocks, stream, map_a, map_b, map_out,
                                        map_residual, map_original, args, M, N, K);
    }
    if (NKS > 0) {
        // units: each row block's column tiles in as many groups as leave every SM one unit (at least one a block); the
        // kernel reads the group count back as grid / row blocks
        int groups = multiprocessors / row_blocks;
        groups = groups < 1 ? 1 : groups > n_blocks ? n_blocks : groups;
        grid = row_blocks * groups < multiprocessors ? row_blocks * groups : multiprocessors;
    }
    return launch_dependent(kernel, dim3(grid), dim3(kGemmThreads), S::kSmemBytes, stream, map_a, map_b, map_out, map_residual,
                            map_original, args, M, N, K);
}

}  // namespace

// Tile widths: one N = 256 MMA a K step where N allows (gate_up's 128 columns hold 256 accumulators, its gate and its
// up), staged in 64-column sub-tiles in three slots (16 KB each, so three 48 KB pipeline stages still fit: against two
// 32 KB slots of 128-column sub-tiles, 1.5-3% faster launches, the stores reading one slot while the next is staged).
// Mixing (two row operands a slot) takes, in place of 256, 192-column tiles, whose 40 KB stages fit four deep beside
// its 96 KB of slots (three at 256). When that leaves fewer tiles
// than SMs (small batches), narrower tiles (128, then 64 columns: more CTAs streaming the weights, deeper pipelines)
// take their place. An fp16 output needs N a multiple of 8 (its rows 16-byte aligned for the TMA maps).
// Where the 256-column tiles fill the SMs (large batches), every GEMM with an fp16 or bf16 output runs as CTA pairs
// (PAIR), the normed-A and norm-epilogue forms excepted: a CTA loads half the B bytes, and a launch at 256 boards takes projection 16.8 -> 16.4 (1152) and 20.3 ->
// 18.9 us (1440), gate_up 24.4 -> 23.8, down 24.1 -> 21.6, attention-out 23.5 -> 19.8 (ten launches a graph). At 64
// boards pairs of 128-column tiles measured slower (gate_up 9.6 -> 10.5 us), so smaller batches keep single CTAs.
cudaError_t gemm(int kind, int epilogue, const void* a, const void* b, const GemmArgs& args, int M, int N, int K, cudaStream_t stream,
                 std::string* error) {
    int device = 0, multiprocessors = 0;
    cudaError_t status = cudaGetDevice(&device);
    if (status == cudaSuccess) status = cudaDeviceGetAttribute(&multiprocessors, cudaDevAttrMultiProcessorCount, device);
    if (status != cudaSuccess) return status;
    const int row_blocks = (M + kBlockM - 1) / kBlockM;
    auto tiles = [&](int bn) { return row_blocks * ((N + bn - 1) / bn); };
    // the widest tile whose count fills the SMs (or the narrowest)
    const int width = tiles(256) >= multiprocessors ? 256 : tiles(128) >= multiprocessors ? 128 : 64;
    if (args.norm_x) {
        // a normed A (NKS = 6 resident K slices: the model width 768); 128-column tiles leave room for 6 pipeline stages
        // beside it, 64-column ones fill the SMs at small batches
        if (kind != 0 || K != kNormedK || (epilogue != kEpiBias && epilogue != kEpiGated)) {
            if (error) *error = "a normed A takes the int8 bias or gated epilogue and K = " + std::to_string(kNormedK);
            return cudaErrorInvalidValue;
        }
        const bool wide = tiles(128) >= multiprocessors;
        if (epilogue == kEpiBias)
            return wide ? launch<0, 128, false, kEpiBias, 64, kNormedSlices>(a, b, args, M, N, K, stream, error)
                        : launch<0, 64, false, kEpiBias, 64, kNormedSlices>(a, b, args, M, N, K, stream, error);
        return wide ? launch<0, 128, true, kEpiGated, 64, kNormedSlices>(a, b, args, M, N, K, stream, error)
                    : launch<0, 64, true, kEpiGated, 64, kNormedSlices>(a, b, args, M, N, K, stream, error);
    }
    if (kind == 0) {
        switch (epilogue) {
            case kEpiBias:
                // 192-column tiles where they pad N less than 256-column ones (the projection at dq 8: 960 against 1024
                // columns; 40 KB stages, four deep): 20.4 -> 19-19.9 us a launch at 256 boards; 128 columns did not gain
                if (width == 256 && (N + 191) / 192 * 192 < (N + 255) / 256 * 256)
                    return launch<0, 192, false, kEpiBias, 64, 0, true>(a, b, args, M, N, K, stream, error);
                if (width == 256) return launch<0, 256, false, kEpiBias, 64, 0, true>(a, b, args, M, N, K, stream, error);
                if (width == 128) return launch<0, 128, false, kEpiBias, 64>(a, b, args, M, N, K, stream, error);
                return launch<0, 64, false, kEpiBias, 64>(a, b, args, M, N, K, stream, error);
            case kEpiBiasQkNorm: {
                const bool dq24 = args.qk_dq == 24;
                const int boundary = dq24 ? 48 : 16;
                if ((args.qk_dq != 8 && args.qk_dq != 16 && !dq24) || args.qk_queries % boundary || args.qk_keys % boundary ||
                    args.qk_keys > N || !args.q_gain || !args.k_gain) {
                    if (error)
                        *error = "the q/k norm epilogue takes heads 8 or 16 wide in blocks starting on 16-column boundaries, or 24 wide "
                                 "on 48-column boundaries, and both gains";
                    return cudaErrorInvalidValue;
                }
                // dq 24: 192-column tiles (8 heads each), so no head leaves its tile, as CTA pairs at every batch
                if (dq24) return launch<0, 192, false, kEpiBiasQkNorm, 64, 0, true>(a, b, args, M, N, K, stream, error);
                if (width == 256 && (N + 191) / 192 * 192 < (N + 255) / 256 * 256)
                    return launch<0, 192, false, kEpiBiasQkNorm, 64, 0, true>(a, b, args, M, N, K, stream, error);
                if (width == 256) return launch<0, 256, false, kEpiBiasQkNorm, 64, 0, true>(a, b, args, M, N, K, stream, error);
                if (width == 128) return launch<0, 128, false, kEpiBiasQkNorm, 64>(a, b, args, M, N, K, stream, error);
                return launch<0, 64, false, kEpiBiasQkNorm, 64>(a, b, args, M, N, K, stream, error);
            }
            case kEpiGated:
                // as pairs, 128-column sub-tiles (two chunks a warp between barriers): 23.8 -> 22.5 us a launch at 256 boards
                if (width == 256) return launch<0, 128, true, kEpiGated, 128, 0, true>(a, b, args, M, N, K, stream, error);
                if (width >= 128 || tiles(128) >= multiprocessors) return launch<0, 128, true, kEpiGated, 64>(a, b, args, M, N, K, stream, error);
                return launch<0, 64, true, kEpiGated>(a, b, args, M, N, K, stream, error);
            case kEpiResidual:
                if (width == 256) return launch<0, 256, false, kEpiResidual, 64, 0, true>(a, b, args, M, N, K, stream, error);
                // one round of 192-column tiles rather than two of 128, as the mixing down
                if (width == 128 && tiles(192) <= multiprocessors) return launch<0, 192, false, kEpiResidual, 64>(a, b, args, M, N, K, stream, error);
                if (width == 128) return launch<0, 128, false, kEpiResidual, 64>(a, b, args, M, N, K, stream, error);
                return launch<0, 64, false, kEpiResidual, 64>(a, b, args, M, N, K, stream, error);
            case kEpiMix:
                // 192 columns also where they take the tiles in one round that 128 would take in two (64 boards: 12.3
                // against 13.8 us a launch)
                if (width == 256) return launch<0, 192, false, kEpiMix, 64, 0, true>(a, b, args, M, N, K, stream, error);
                if (width == 128 && tiles(192) <= multiprocessors) return launch<0, 192, false, kEpiMix, 64>(a, b, args, M, N, K, stream, error);
                if (width == 128) return launch<0, 128, false, kEpiMix, 64>(a, b, args, M, N, K, stream, error);
                return launch<0, 64, false, kEpiMix, 64>(a, b, args, M, N, K, stream, error);
            case kEpiInt32: return launch<0, 128, false, kEpiInt32>(a, b, args, M, N, K, stream, error);
            case kEpiScaleBf16:
                if (width == 256) return launch<0, 256, false, kEpiScaleBf16, 64, 0, true>(a, b, args, M, N, K, stream, error);
                if (width == 128) return launch<0, 128, false, kEpiScaleBf16, 64>(a, b, args, M, N, K, stream, error);
                return launch<0, 64, false, kEpiScaleBf16, 64>(a, b, args, M, N, K, stream, error);
            default: break;
        }
    } else {
        switch (epilogue) {
            case kEpiLinearF16:
                if (width == 256) return launch<1, 256, false, kEpiLinearF16, 64, 0, true>(a, b, args, M, N, K, stream, error);
                // 192 columns where they take the tiles in one round that 128 would take in two, as single CTAs (64 boards:
                // the forward 1.818 -> 1.798 ms; as CTA pairs 1.807)
                if (width == 128 && tiles(192) <= multiprocessors) return launch<1, 192, false, kEpiLinearF16, 64>(a, b, args, M, N, K, stream, error);
                if (width == 128) return launch<1, 128, false, kEpiLinearF16, 64>(a, b, args, M, N, K, stream, error);
                return launch<1, 64, false, kEpiLinearF16, 64>(a, b, args, M, N, K, stream, error);
            case kEpiLinearF32:
                if (width == 256) return launch<1, 256, false, kEpiLinearF32, 256, 0, true>(a, b, args, M, N, K, stream, error);
                // one round of 192-column tiles rather than two of 128 (64 boards: 19.9 -> 17.2 us a launch)
                if (width == 128 && tiles(192) <= multiprocessors) return launch<1, 192, false, kEpiLinearF32, 192>(a, b, args, M, N, K, stream, error);
                return launch<1, 128, false, kEpiLinearF32>(a, b, args, M, N, K, stream, error);
            case kEpiGatedF16:
                if (width == 256) return launch<1, 128, true, kEpiGatedF16, 64, 0, true>(a, b, args, M, N, K, stream, error);
                if (width >= 128 || tiles(128) >= multiprocessors) return launch<1, 128, true, kEpiGatedF16, 64>(a, b, args, M, N, K, stream, error);
                return launch<1, 64, true, kEpiGatedF16>(a, b, args, M, N, K, stream, error);
            case kEpiMixF16:
                if (width == 256) return launch<1, 192, false, kEpiMixF16, 64, 0, true>(a, b, args, M, N, K, stream, error);
                if (width == 128) return launch<1, 128, false, kEpiMixF16, 64>(a, b, args, M, N, K, stream, error);
                return launch<1, 64, false, kEpiMixF16, 64>(a, b, args, M, N, K, stream, error);
            case kEpiLinearNorm:
                if (N % 256 != 0 || N / 256 > kMaxCluster || !args.norm_q || !args.norm_scale || !args.norm_gain) {
                    if (error) *error = "the norm epilogue takes N a multiple of 256 up to " + std::to_string(256 * kMaxCluster) + " and its outputs";
                    return cudaErrorInvalidValue;
                }
                return launch<1, 256, false, kEpiLinearNorm, 128>(a, b, args, M, N, K, stream, error);
            default: break;
        }
    }
    if (error) *error = "no GEMM for this kind and epilogue";
    return cudaErrorInvalidValue;
}

}  // namespace fry
