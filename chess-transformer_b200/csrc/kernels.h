// Internal launch API of the Fry kernels (C++). The C ABI in abi.cu wraps these; include/fry_b200.h declares it.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

namespace fry {

// GEMM epilogues. The int8 ones follow model/int8_cuda.py:163-178 (EPI 0-3 there); the fp16 ones
// model/fused_blocks.py:208-225 without the gate.
enum GemmEpilogue : int {
    kEpiBias = 0,       // int8: fp16(fma(acc * xs, ws, bias))
    kEpiGated = 1,      // int8: fp16((g * sigmoid(g)) * u), weight rows = gate rows then up rows
    kEpiResidual = 2,   // int8: fp16(fma(acc * xs, ws, residual))
    kEpiMix = 3,        // int8: the residual sum rounded to fp16, then fp16(fma(stream, rs, original * is))
    kEpiInt32 = 4,      // int8: the raw int32 sums
    kEpiLinearF16 = 5,  // fp16: fp16((acc + bias) + residual), bias and residual optional
    kEpiLinearF32 = 6,  // fp16: fp32 acc + fp32 bias (optional)
    kEpiLinearNorm = 7, // fp16: as kEpiLinearF16, then norm_quant of each output row into norm_q / norm_scale (a cluster of
                        // the N / 256 CTAs of a row block sums the rows' squares through distributed shared memory)
    // the fp16 blocks' linears (model/fused_blocks.py:209-225), on fp32 sums:
    kEpiGatedF16 = 8,   // fp16: fp16((g * sigmoid(g)) * u), weight rows = gate rows then up rows
    kEpiMixF16 = 9,     // fp16: (acc + bias) + residual rounded to fp16, then fp16(fma(stream, rs, original * is))
    kEpiScaleBf16 = 10, // int8: bf16((acc * xs) * ws), the scaled GEMM of the isolated-kernel benchmark (no reference op)
    kEpiBiasQkNorm = 11,// int8: kEpiBias, then the attention's q and k RMSNorm with gains on the query and key columns (qk_*)
};

struct GemmArgs {
    const float* x_scale = nullptr;          // [M]
    const float* w_scale = nullptr;          // [N] ([2N] gated)
    const uint16_t* bias = nullptr;          // fp16 [N]
    const float* bias_f32 = nullptr;         // fp32 [N]
    const uint16_t* residual = nullptr;      // fp16 [M, N]
    const uint16_t* original = nullptr;      // fp16 [M, N]
    const uint16_t* residual_scale = nullptr;  // fp16 scalar
    const uint16_t* input_scale = nullptr;     // fp16 scalar
    void* out = nullptr;                     // [M, N]
    // Normed A (kind 0, bias or gated epilogue, K = 768): A is norm_quant(norm_x) with norm_gain and norm_eps, made in
    // the GEMM's prologue; `a` and x_scale are then unused.
    const uint16_t* norm_x = nullptr;        // fp16 [M, K]
    const uint16_t* norm_gain = nullptr;     // fp16 [K]
    float norm_eps = 0.0f;
    // B is a weight that no kernel launched before this one writes: its first stages load before the wait for the
    // earlier kernels (programmatic dependent launch), overlapping their tail
    bool b_constant = false;
    // kEpiLinearNorm: the int8 rows [M, N] and their scales [M] of norm_quant(out) with norm_gain and norm_eps
    int8_t* norm_q = nullptr;
    float* norm_scale = nullptr;
    // kEpiBiasQkNorm: columns [0, qk_queries) are query heads and [qk_queries, qk_keys) key heads, qk_dq (8, 16 or 24) wide,
    // each RMS-normalised (eps norm_eps) and scaled by q_gain / k_gain [qk_dq] after the fp16 rounding
    const uint16_t* q_gain = nullptr;
    const uint16_t* k_gain = nullptr;
    int qk_dq = 0, qk_queries = 0, qk_keys = 0;
};

// kind 0: int8 A [M, K], B [N, K] (gated: [2N, K]); kind 1: fp16 A [M, K], B [N, K].
cudaError_t gemm(int kind, int epilogue, const void* a, const void* b, const GemmArgs& args, int M, int N, int K, cudaStream_t stream,
                 std::string* error);

// Row kernels (rows.cu).
cudaError_t norm_quant(const uint16_t* x, const uint16_t* original, const uint16_t* residual_scale, const uint16_t* input_scale,
                       const uint16_t* gain, float eps, uint16_t* mixed, int8_t* q, float* scale, int M, int D, cudaStream_t stream);
cudaError_t rms_norm_f16(const uint16_t* x, const uint16_t* gain, float eps, uint16_t* y, int M, int D, cudaStream_t stream);
// An fp16 block mixing its own input as torch's fp16 ops do (model/fused_blocks.py:346-347): out = fp16(fp16(rs * x) +
// fp16(is * original)), elementwise over [M, D]; out may alias x.
cudaError_t mix_input_f16(const uint16_t* x, const uint16_t* original, const uint16_t* residual_scale, const uint16_t* input_scale,
                          uint16_t* out, int M, int D, cudaStream_t stream);
cudaError_t rotate_quant(const uint16_t* h, int8_t* q, float* scale, int M, int hidden, int width, cudaStream_t stream);
// Lean lanes (engine/inference.py:94-100,130-135; engine/selfplay_rs/src/lib.rs:330-333): a board is a row of
// kLeanRow bytes, its 70 token bytes then kLeanColumns int16 answer columns, and its answer those columns of its row.
constexpr int kLeanColumns = 219, kLeanRow = 70 + 2 * kLeanColumns;
cudaError_t board_embedding_lean(const uint8_t* lean_rows, const uint16_t* embed, const uint16_t* position, const uint16_t* table,
                                 uint16_t* out, int B, int D, cudaStream_t stream);
cudaError_t board_embedding(const int64_t* boards, const uint16_t* embed, const uint16_t* position, const uint16_t* table,
                            uint16_t* out, int B, int D, cudaStream_t stream);
// Each square's 23 feature rows of the table (SquareFeatures.indices with the features' first rows added,
// model/model.py:134-169): boards int64 [B, 70] -> rows int32 [B, 64, 23].
cudaError_t square_feature_rows(const int64_t* boards, int32_t* rows, int B, cudaStream_t stream);

// Template attention (attention.cu).
// paired [64][64][8] fp16: templates[t][i][j] at paired[i][j][t]
cudaError_t pair_templates(const uint16_t* templates, uint16_t* paired, cudaStream_t stream);
// qk_normed: the projected rows' query and key columns are already normalised with their gains (kEpiBiasQkNorm; dq 8,
// 16 or 24)
cudaError_t template_attention(const uint16_t* projected, const uint16_t* paired, const uint16_t* q_gain, const uint16_t* k_gain,
                               uint16_t* out, int B, int heads, int kv_heads, int dq, int dv, int templates_count, float eps,
                               cudaStream_t stream, std::string* error, bool qk_normed = false);

// Attention over 64-token sequences with 64-wide heads, bf16 (attention64.cu): q, k, v, out [B, 64, heads * 64].
cudaError_t attention64(const uint16_t* q, const uint16_t* k, const uint16_t* v, uint16_t* out, int B, int heads, cudaStream_t stream,
                        std::string* error);

// Heads (heads.cu).
struct HeadWeights {
    const uint16_t* ln_gain;         // fp16 [d]
    const uint16_t* a_weight;        // fp16 [d, d]: row n of (W_f^T W_t / sqrt d)^T, K-major for the GEMM
    const float* a_bias;             // fp32 [d]
    const float* narrow_weight;      // fp32 [21, d]: s, 4 promotions, 16 board-down rows
    const float* narrow_bias;        // fp32 [21]
    const float* hidden_weight;      // fp32 [d, 1120]
    const float* hidden_bias;        // fp32 [d]
    const float* out_weight;         // fp32 [bins, d]
    const float* out_bias;           // fp32 [bins]
    int bins;
};
// The heads' scratch, each region 256-byte aligned: y fp16 and a fp32 per token row, narrow (24 floats a token row), the
// eval head's GELU'd inputs (70 x 16 a board), its split-K partial sums (up to kEvalSplitsMax splits of B x max(D, 256)),
// its hidden units [B, D] and its value logits [B, up to 256 bins].
constexpr int kEvalSplitsMax = 8;
struct HeadsWorkspace {
    size_t y, a, narrow, eval_in, partial, hidden, logits, total;
    static constexpr size_t up(size_t bytes) { return (bytes + 255) / 256 * 256; }
    constexpr HeadsWorkspace(size_t B, size_t D)
        : y(0), a(up(B * 70 * D * 2)), narrow(a + up(B * 70 * D * 4)), eval_in(narrow + up(B * 70 * 24 * 4)),
          partial(eval_in + up(B * 70 * 16 * 4)), hidden(partial + up(kEvalSplitsMax * B * (D > 256 ? D : 256) * 4)),
          logits(hidden + up(B * D * 4)), total(logits + up(B * 256 * 4)) {}
};
constexpr size_t heads_workspace_bytes_of(size_t B, size_t D) { return HeadsWorkspace(B, D).total; }
size_t heads_workspace_bytes(int B, int D);
// lean_rows / lean_answers (optional): each board's answer columns gathered from its row into lean_answers [B, 219]
cudaError_t heads(const uint16_t* stream_x, const HeadWeights& w, float eps, float* rows, void* workspace, size_t workspace_bytes, int B,
                  int D, cudaStream_t stream, std::string* error, const uint8_t* lean_rows = nullptr, float* lean_answers = nullptr);

// GPTQ (engine/quantization.py:76-99): weight fp64 [N, K], hessian fp64 [K, K] -> q int8 [N, K], scale fp32 [N]. The
// workspace holds fp64 copies of both ([K, K] twice, [N, K]), a block's errors [N, 128], the fp64 scales and the dead flags.
struct GptqWorkspace {
    size_t hessian, inverse, weight, errors, scale, dead, total;
    GptqWorkspace(size_t N, size_t K);
};
cudaError_t gptq(const double* weight, const double* hessian, int N, int K, int8_t* q, float* scale, void* workspace,
                 size_t workspace_bytes, cudaStream_t stream, std::string* error);
// H [K, K] += x^T x, x [rows, K], fp64 (the input sums GPTQ's Hessians are made of)
cudaError_t hessian_accumulate(const double* x, int rows, int K, double* H, cudaStream_t stream, std::string* error);

}  // namespace fry
