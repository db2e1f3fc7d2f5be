// Scaled dot-product attention over 64-token sequences with 64-wide heads in bf16: out = softmax(q k^T / 8) v for each
// (sequence, head). This is the isolated attention kernel of the benchmark's microbench configuration (seq 64, head_dim
// 64, bf16 q/k/v); Fry's own blocks run the template attention of attention.cu, whose reference test it follows in
// checking (model/fused_blocks.py:54-97 is the reference's kernel of the same shape family; its test compares against
// fp32 torch at atol 1e-2, tests/test_attention_cuda.py:63-71).
//
// Layout: q, k, v and out are [B, 64, heads * 64] bf16 row-major, the rows of a projection GEMM's output (token-major,
// heads side by side). One CTA per (head, sequence) and four warps, each taking 16 query rows:
//  - one thread loads the head's 64 x 64 tiles of q, k and v with TMA (2-D tiled, 128-byte swizzle: 16-byte unit u of
//    row r at u ^ (r % 8)), all three completing on one mbarrier (a bounded wait);
//  - each warp reads its q rows' A fragments and the k and v B fragments with ldmatrix (the swizzle spreads the 8 rows
//    of each 8x8 matrix over all banks), forms its 16 x 64 scores with mma.sync m16n8k16 (bf16 in, fp32 sums), takes the
//    softmax in registers (quad shuffles for the row max and sum, 2^x with log2(e)/8 folded in), rounds the
//    probabilities to bf16 as the A fragments of P.V and divides the fp32 sums by the unrounded row total;
//  - the warp writes its 16 output rows in bf16 over its own q rows (no other warp reads them), and one TMA store
//    writes the 64 x 64 tile.
// The work is 1 MFLOP per (sequence, head) on 32 KB of HBM traffic: HBM-bound, so the tensor steps stay on mma.sync in
// registers; what matters is enough CTAs in flight per SM (8, at 25 KB of shared memory each) to cover the loads.
#include <string>

#include "common.cuh"
#include "kernels.h"

namespace fry {

constexpr int kSeq64 = 64, kHead64 = 64;
constexpr int kTile64Bytes = kSeq64 * kHead64 * 2;  // one head's 64 rows of 128 bytes
constexpr int kAttention64Threads = 128;
constexpr int kAttention64Smem = 3 * kTile64Bytes + 64 + 1024;  // q, k, v tiles, the barrier, and room to align to 1024

FRY_DEVICE void mma_bf16(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
FRY_DEVICE void ldmatrix_x4(uint32_t address, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(address));
}
FRY_DEVICE void ldmatrix_x4_trans(uint32_t address, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(address));
}
// byte offset of 16-byte unit `unit` of row `row` in a tile of 128-byte rows in the 128-byte swizzle
FRY_DEVICE uint32_t swizzled128(int row, int unit) { return static_cast<uint32_t>(row * 128 + ((unit ^ (row & 7)) << 4)); }
FRY_DEVICE float quad_max64(float v) {
    v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 1));
    return fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 2));
}
FRY_DEVICE float quad_sum64(float v) {
    v += __shfl_xor_sync(0xffffffffu, v, 1);
    return v + __shfl_xor_sync(0xffffffffu, v, 2);
}

// scale_log2 = log2(e) / sqrt(64): softmax(s / 8) = 2^(s scale_log2 - max) / sum
__global__ void __launch_bounds__(kAttention64Threads) attention64_kernel(const __grid_constant__ CUtensorMap map_q,
                                                                         const __grid_constant__ CUtensorMap map_k,
                                                                         const __grid_constant__ CUtensorMap map_v,
                                                                         const __grid_constant__ CUtensorMap map_out, float scale_log2) {
    extern __shared__ uint8_t raw[];
    // the tiles start on a 1024-byte boundary, as the swizzle's 8-row atoms need
    const uint32_t base = (smem_addr(raw) + 1023u) & ~1023u;
    uint8_t* q_tile = raw + (base - smem_addr(raw));
    uint8_t* k_tile = q_tile + kTile64Bytes;
    uint8_t* v_tile = k_tile + kTile64Bytes;
    uint64_t* full = reinterpret_cast<uint64_t*>(v_tile + kTile64Bytes);
    const int x = blockIdx.x * kHead64, y = blockIdx.y * kSeq64;  // the head's columns, the sequence's first row
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;

    if (threadIdx.x == 0) {
        mbar_init(full, 1);
        fence_barrier_init();
        prefetch_tensor_map(&map_q);
        prefetch_tensor_map(&map_k);
        prefetch_tensor_map(&map_v);
    }
    __syncthreads();
    grid_dependency_start();  // q, k and v may come from the kernel before
    if (threadIdx.x == 0) {
        mbar_arrive_expect_tx(full, 3 * kTile64Bytes);
        tma_load_2d(q_tile, &map_q, full, x, y);
        tma_load_2d(k_tile, &map_k, full, x, y);
        tma_load_2d(v_tile, &map_v, full, x, y);
    }
    if (!mbar_wait(full, 0, 80)) return;  // recorded in the status word
    const uint32_t q_base = smem_addr(q_tile), k_base = smem_addr(k_tile), v_base = smem_addr(v_tile);

    // the warp's 16 query rows as A fragments, one per 16 dims: matrices (rows 0-7 | 8-15) x (dims 0-7 | 8-15)
    uint32_t qa[4][4];
    const int q_row = warp * 16 + (lane & 15);
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) ldmatrix_x4(q_base + swizzled128(q_row, 2 * kk + (lane >> 4)), qa[kk]);

    // scores: key tiles j (keys 8j .. 8j + 7); one ldmatrix gives two key tiles' B fragments for 16 dims
    float s[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.0f;
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
        for (int jp = 0; jp < 4; ++jp) {
            uint32_t b[4];
            const int key = 16 * jp + (lane & 7) + ((lane >> 4) << 3);
            ldmatrix_x4(k_base + swizzled128(key, 2 * kk + ((lane >> 3) & 1)), b);
            mma_bf16(s[2 * jp], qa[kk], b[0], b[1]);
            mma_bf16(s[2 * jp + 1], qa[kk], b[2], b[3]);
        }
    }

    // softmax of rows g (s[j][0..1]) and g + 8 (s[j][2..3]) over the 64 keys, a row's keys spread over a quad
    float top0 = s[0][0], top1 = s[0][2];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        top0 = fmaxf(top0, fmaxf(s[j][0], s[j][1]));
        top1 = fmaxf(top1, fmaxf(s[j][2], s[j][3]));
    }
    top0 = quad_max64(top0) * scale_log2;
    top1 = quad_max64(top1) * scale_log2;
    float sum0 = 0.0f, sum1 = 0.0f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        s[j][0] = ex2_approx_ftz(__fmaf_rn(s[j][0], scale_log2, -top0));
        s[j][1] = ex2_approx_ftz(__fmaf_rn(s[j][1], scale_log2, -top0));
        s[j][2] = ex2_approx_ftz(__fmaf_rn(s[j][2], scale_log2, -top1));
        s[j][3] = ex2_approx_ftz(__fmaf_rn(s[j][3], scale_log2, -top1));
        sum0 += s[j][0] + s[j][1];
        sum1 += s[j][2] + s[j][3];
    }
    sum0 = quad_sum64(sum0);
    sum1 = quad_sum64(sum1);

    // P.V: the probabilities of keys 16kk .. 16kk + 15 are the A fragment of step kk; the values' B fragments come
    // transposed, two 8-dim output tiles a load
    float o[8][4];
#pragma unroll
    for (int d = 0; d < 8; ++d) o[d][0] = o[d][1] = o[d][2] = o[d][3] = 0.0f;
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
        const uint32_t pa[4] = {pack_bf162_rn(s[2 * kk][0], s[2 * kk][1]), pack_bf162_rn(s[2 * kk][2], s[2 * kk][3]),
                                pack_bf162_rn(s[2 * kk + 1][0], s[2 * kk + 1][1]), pack_bf162_rn(s[2 * kk + 1][2], s[2 * kk + 1][3])};
#pragma unroll
        for (int dp = 0; dp < 4; ++dp) {
            uint32_t b[4];
            ldmatrix_x4_trans(v_base + swizzled128(16 * kk + (lane & 15), 2 * dp + (lane >> 4)), b);
            mma_bf16(o[2 * dp], pa, b[0], b[1]);
            mma_bf16(o[2 * dp + 1], pa, b[2], b[3]);
        }
    }

    // the warp's rows, normalised and rounded to bf16, over its own q rows (its fragments are in registers)
    const float inverse0 = div_full(1.0f, sum0), inverse1 = div_full(1.0f, sum1);
    const int row0 = warp * 16 + g, row1 = row0 + 8;
#pragma unroll
    for (int d = 0; d < 8; ++d) {
        *reinterpret_cast<uint32_t*>(q_tile + swizzled128(row0, d) + 4 * t) = pack_bf162_rn(o[d][0] * inverse0, o[d][1] * inverse0);
        *reinterpret_cast<uint32_t*>(q_tile + swizzled128(row1, d) + 4 * t) = pack_bf162_rn(o[d][2] * inverse1, o[d][3] * inverse1);
    }
    fence_proxy_async_shared();  // the staged rows, visible to the TMA store
    __syncthreads();
    if (threadIdx.x == 0) {
        tma_store_2d(&map_out, q_tile, x, y);
        bulk_commit();
        bulk_wait_read_all();  // the tile is read out before the CTA's shared memory goes
    }
}

namespace {

// a [rows, cols] bf16 row-major tensor as a TMA map with 64 x 64 boxes in the 128-byte swizzle
bool attention64_map(CUtensorMap* map, const void* base, int cols, int rows, std::string* error) {
    using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*, const cuuint64_t*,
                                     const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                     CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
    static EncodeTiled encode = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* symbol = nullptr;
        cudaDriverEntryPointQueryResult found;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &symbol, cudaEnableDefault, &found) == cudaSuccess &&
            found == cudaDriverEntryPointSuccess)
            encode = reinterpret_cast<EncodeTiled>(symbol);
    });
    if (!encode) {
        if (error) *error = "the CUDA driver has no cuTensorMapEncodeTiled";
        return false;
    }
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols) * 2};
    const cuuint32_t box[2] = {kHead64, kSeq64};
    const cuuint32_t element_strides[2] = {1, 1};
    const CUresult result = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, element_strides,
                                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (result != CUDA_SUCCESS) {
        if (error) *error = "cuTensorMapEncodeTiled (bf16 attention tile) failed with CUresult " + std::to_string(static_cast<int>(result));
        return false;
    }
    return true;
}

}  // namespace

cudaError_t attention64(const uint16_t* q, const uint16_t* k, const uint16_t* v, uint16_t* out, int B, int heads, cudaStream_t stream,
                        std::string* error) {
    if (B <= 0) return cudaSuccess;
    if (B > 65535 || heads <= 0 || heads > 1024) {
        if (error) *error = "the attention takes 1 to 65535 sequences of 1 to 1024 heads";
        return cudaErrorInvalidValue;
    }
    const int cols = heads * kHead64, rows = B * kSeq64;
    CUtensorMap map_q, map_k, map_v, map_out;
    if (!attention64_map(&map_q, q, cols, rows, error) || !attention64_map(&map_k, k, cols, rows, error) ||
        !attention64_map(&map_v, v, cols, rows, error) || !attention64_map(&map_out, out, cols, rows, error))
        return cudaErrorInvalidValue;
    const cudaError_t attribute = ensure_smem(reinterpret_cast<const void*>(attention64_kernel), kAttention64Smem);
    if (attribute != cudaSuccess) return attribute;
    const float scale_log2 = 1.4426950408889634f / 8.0f;  // log2(e) / sqrt(64)
    return launch_dependent(attention64_kernel, dim3(heads, B), dim3(kAttention64Threads), kAttention64Smem, stream, map_q, map_k, map_v,
                            map_out, scale_log2);
}

}  // namespace fry
