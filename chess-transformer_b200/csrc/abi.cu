// The C ABI (include/fry_b200.h): argument checks on the host, then the kernels of gemm.cu, rows.cu, attention.cu and
// heads.cu on the caller's stream. fry_forward runs the whole int8 network: the block sequence of `Int8Block.forward`
// (model/int8_blocks.py:274-288) with `link_input_mixes` (model/fused_blocks.py:358-363), then the heads.
#include <cstdio>
#include <string>

#include "../../include/fry_b200.h"
#include "common.cuh"
#include "kernels.h"

namespace {

thread_local std::string g_last_error;

int fail(int code, const std::string& message) {
    g_last_error = message;
    return code;
}

int check(cudaError_t status, const std::string& what, const std::string& detail = "") {
    if (status == cudaSuccess) {
        g_last_error.clear();
        return FRY_OK;
    }
    std::string message = what + ": " + cudaGetErrorString(status);
    if (!detail.empty()) message += " (" + detail + ")";
    return fail(status == cudaErrorInvalidValue && !detail.empty() ? FRY_ERROR_SHAPE : FRY_ERROR_CUDA, message);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

cudaStream_t as_stream(void* stream) { return static_cast<cudaStream_t>(stream); }

size_t round_up(size_t bytes) { return (bytes + 255) / 256 * 256; }

int projection_rows(const FryNetwork* n, int dq) {
    return (n->heads + n->kv_heads) * dq + n->kv_heads * n->dv + n->heads * n->templates_count;
}

constexpr int kAnswerWidth = 1969;  // 1968 move logits, then the expected score
constexpr uint64_t kMaxWaitLimitNs = 60000000000ull;  // the largest wait limit fry_set_wait_limit_ns takes: 60 s

// The forward on boards (int64 [B, 70]) or on lean lanes' rows (uint8 [B, 508]: tokens, then the answer columns that
// lean_answers [B, 219] gathers from rows), in the caller's workspace of fry_forward_workspace_bytes.
int run_forward(const FryNetwork* n, const int64_t* boards, const uint8_t* lean_rows, int B, float* rows, float* lean_answers,
                void* workspace, size_t workspace_bytes, void* stream) {
    if (!n || B < 0) return fail(FRY_ERROR_SHAPE, "fry_forward needs a network and B >= 0");
    if (B == 0) return check(cudaSuccess, "");
    if (workspace_bytes < fry_forward_workspace_bytes(n, B))
        return fail(FRY_ERROR_SHAPE, "fry_forward's workspace is smaller than fry_forward_workspace_bytes");
    if (!aligned16(workspace)) return fail(FRY_ERROR_SHAPE, "fry_forward needs a 16-byte aligned workspace");
    const cudaStream_t s = as_stream(stream);
    const int D = n->d_model, M = B * 70;
    uint8_t* cursor = static_cast<uint8_t*>(workspace);
    auto take = [&](size_t bytes) {
        uint8_t* p = cursor;
        cursor += round_up(bytes);
        return p;
    };
    int widest = 0;
    for (int i = 0; i < n->layers; ++i) {
        const int r = projection_rows(n, n->blocks[i].dq);
        widest = r > widest ? r : widest;
    }
    const int q_width = D > n->down_width ? D : n->down_width;
    uint16_t* original = reinterpret_cast<uint16_t*>(take(static_cast<size_t>(M) * D * 2));
    uint16_t* x = reinterpret_cast<uint16_t*>(take(static_cast<size_t>(M) * D * 2));
    uint16_t* attended = reinterpret_cast<uint16_t*>(take(static_cast<size_t>(M) * D * 2));
    int8_t* q = reinterpret_cast<int8_t*>(take(static_cast<size_t>(M) * q_width));
    float* scale = reinterpret_cast<float*>(take(static_cast<size_t>(M) * 4));
    uint16_t* projected = reinterpret_cast<uint16_t*>(take(static_cast<size_t>(M) * widest * 2));
    uint16_t* hidden = reinterpret_cast<uint16_t*>(take(static_cast<size_t>(M) * n->hidden * 2));
    const size_t heads_bytes = fry::heads_workspace_bytes(B, D);
    void* heads_workspace = take(heads_bytes);

    // ln1 and ln2 run as their own kernels. Fused into a neighbouring GEMM they measured slower: in the int8 GEMM's prologue
    // (fry_int8_linear_normed) no faster at 256 boards and slower at small batches, where each CTA of a row block repeats
    // the block's norm; in the attention-out GEMM's epilogue (fry_linear_norm_quant) slower at every batch, its clusters
    // of 3 CTAs taking up to 4 row blocks where single CTAs take 3 tiles, and its cluster exchange adding to each tile
    std::string detail;
    cudaError_t status = lean_rows ? fry::board_embedding_lean(lean_rows, n->embed, n->position, n->table, original, B, D, s)
                                   : fry::board_embedding(boards, n->embed, n->position, n->table, original, B, D, s);
    if (status != cudaSuccess) return check(status, "fry_forward: embedding");
    for (int i = 0; i < n->layers; ++i) {
        const FryBlock& b = n->blocks[i];
        const std::string where = "fry_forward: block " + std::to_string(i);
        const bool fp16 = b.precision == FRY_BLOCK_FP16;
        // link_input_mixes: a block mixes its own input when first or after a block of the other precision; its down
        // mixes the next block's when that one is of its own precision
        const bool mixes_own = i == 0 || n->blocks[i - 1].precision != b.precision;
        const bool mixes_next = i + 1 < n->layers && n->blocks[i + 1].precision == b.precision;
        const int rows_p = projection_rows(n, b.dq);
        // an int8 block whose query/key heads are 8 or 16 wide has its projection's epilogue apply the attention's q and
        // k RMSNorm (the same bits as the attention's own), so the attention copies them. At 24 wide the attention
        // normalises them itself: the epilogue that does it for 24-wide heads (fry_int8_linear_qk_norm) measured a
        // slower forward, 4.68 -> 4.74 ms at 256 boards.
        const bool qk_normed = !fp16 && (b.dq == 8 || b.dq == 16) && (n->heads * b.dq) % 16 == 0 && ((n->heads + n->kv_heads) * b.dq) % 16 == 0;
        fry::GemmArgs projection;
        projection.bias = b.projection_bias;
        projection.out = projected;
        projection.b_constant = true;
        if (fp16) {
            // FusedBlock (model/fused_blocks.py:344-354): fp16 norms and linears
            if (mixes_own) {
                status = fry::mix_input_f16(i == 0 ? original : x, original, b.residual_scale, b.input_scale, x, M, D, s);
                if (status != cudaSuccess) return check(status, where + " input mix");
            }
            status = fry::rms_norm_f16(x, b.ln1, n->eps, attended, M, D, s);  // attended holds ln1's rows until the attention
            if (status != cudaSuccess) return check(status, where + " ln1");
            status = fry::gemm(1, fry::kEpiLinearF16, attended, b.projection, projection, M, rows_p, D, s, &detail);
        } else {
            // ln1, mixing the block's own input first where it does
            status = !mixes_own ? fry::norm_quant(x, nullptr, nullptr, nullptr, b.ln1, n->eps, nullptr, q, scale, M, D, s)
                                : fry::norm_quant(i == 0 ? original : x, original, b.residual_scale, b.input_scale, b.ln1, n->eps, x, q, scale,
                                                  M, D, s);
            if (status != cudaSuccess) return check(status, where + " ln1");
            projection.x_scale = scale;
            projection.w_scale = b.projection_scale;
            if (qk_normed) {
                projection.q_gain = b.q_gain;
                projection.k_gain = b.k_gain;
                projection.qk_dq = b.dq;
                projection.qk_queries = n->heads * b.dq;
                projection.qk_keys = (n->heads + n->kv_heads) * b.dq;
                projection.norm_eps = n->eps;
            }
            status = fry::gemm(0, qk_normed ? fry::kEpiBiasQkNorm : fry::kEpiBias, q, b.projection, projection, M, rows_p, D, s, &detail);
        }
        if (status != cudaSuccess) return check(status, where + " projection", detail);
        status = fry::template_attention(projected, n->templates, b.q_gain, b.k_gain, attended, B, n->heads, n->kv_heads, b.dq, n->dv,
                                         n->templates_count, n->eps, s, &detail, qk_normed);
        if (status != cudaSuccess) return check(status, where + " attention", detail);
        fry::GemmArgs combine;
        combine.bias = b.combine_heads_bias;
        combine.residual = x;
        combine.out = x;
        combine.b_constant = true;
        status = fry::gemm(1, fry::kEpiLinearF16, attended, b.combine_heads, combine, M, D, D, s, &detail);
        if (status != cudaSuccess) return check(status, where + " combine_heads", detail);
        fry::GemmArgs gate_up;
        gate_up.out = hidden;
        gate_up.b_constant = true;
        fry::GemmArgs down;
        down.residual = x;
        down.out = x;
        down.b_constant = true;
        if (mixes_next) {
            down.original = original;
            down.residual_scale = n->blocks[i + 1].residual_scale;
            down.input_scale = n->blocks[i + 1].input_scale;
        }
        if (fp16) {
            status = fry::rms_norm_f16(x, b.ln2, n->eps, attended, M, D, s);
            if (status != cudaSuccess) return check(status, where + " ln2");
            status = fry::gemm(1, fry::kEpiGatedF16, attended, b.gate_up, gate_up, M, n->hidden, D, s, &detail);
            if (status != cudaSuccess) return check(status, where + " gate_up", detail);
            status = fry::gemm(1, mixes_next ? fry::kEpiMixF16 : fry::kEpiLinearF16, hidden, b.down, down, M, D, n->hidden, s, &detail);
            if (status != cudaSuccess) return check(status, where + " down", detail);
            continue;
        }
        status = fry::norm_quant(x, nullptr, nullptr, nullptr, b.ln2, n->eps, nullptr, q, scale, M, D, s);
        if (status != cudaSuccess) return check(status, where + " ln2");
        gate_up.x_scale = scale;
        gate_up.w_scale = b.gate_up_scale;
        status = fry::gemm(0, fry::kEpiGated, q, b.gate_up, gate_up, M, n->hidden, D, s, &detail);
        if (status != cudaSuccess) return check(status, where + " gate_up", detail);
        status = fry::rotate_quant(hidden, q, scale, M, n->hidden, n->down_width, s);
        if (status != cudaSuccess) return check(status, where + " rotate_quant");
        down.x_scale = scale;
        down.w_scale = b.down_scale;
        status = fry::gemm(0, mixes_next ? fry::kEpiMix : fry::kEpiResidual, q, b.down, down, M, D, n->down_width, s, &detail);
        if (status != cudaSuccess) return check(status, where + " down", detail);
    }
    const FryHeads& h = n->head_weights;
    fry::HeadWeights w{h.ln_gain, h.a_weight, h.a_bias, h.narrow_weight, h.narrow_bias, h.hidden_weight, h.hidden_bias, h.out_weight,
                       h.out_bias, h.bins};
    status = fry::heads(x, w, n->eps, rows, heads_workspace, heads_bytes, B, D, s, &detail, lean_rows, lean_answers);
    return check(status, "fry_forward: heads", detail);
}

}  // namespace

extern "C" {

const char* fry_last_error(void) { return g_last_error.c_str(); }

const char* fry_version(void) { return "fry_b200 0.1 sm_100a"; }

int fry_device_status(int* code, int* where, int clear) {
    int host[2] = {0, 0};
    cudaError_t status = cudaMemcpyFromSymbol(host, fry::g_status, sizeof(host));
    if (status == cudaSuccess && clear) {
        const int zero[2] = {0, 0};
        status = cudaMemcpyToSymbol(fry::g_status, zero, sizeof(zero));
    }
    if (code) *code = host[0];
    if (where) *where = host[1];
    return check(status, "fry_device_status");
}

int fry_set_wait_limit_ns(uint64_t limit_ns) {
    if (limit_ns < 1000 || limit_ns > kMaxWaitLimitNs)
        return fail(FRY_ERROR_SHAPE, "fry_set_wait_limit_ns takes 1 us to 60 s, got " + std::to_string(limit_ns) + " ns");
    return check(cudaMemcpyToSymbol(fry::g_wait_limit_ns, &limit_ns, sizeof(limit_ns)), "fry_set_wait_limit_ns");
}

int fry_wait_limit_ns(uint64_t* limit_ns) {
    if (!limit_ns) return fail(FRY_ERROR_SHAPE, "fry_wait_limit_ns needs somewhere to write the limit");
    return check(cudaMemcpyFromSymbol(limit_ns, fry::g_wait_limit_ns, sizeof(*limit_ns)), "fry_wait_limit_ns");
}

int fry_wait_probe(void* stream) { return check(fry::wait_probe(as_stream(stream)), "fry_wait_probe"); }

int fry_int8_linear(const int8_t* x, const float* x_scale, const int8_t* weight, const float* weight_scale, const uint16_t* bias,
                    const uint16_t* residual, const uint16_t* original, const uint16_t* residual_scale, const uint16_t* input_scale,
                    uint16_t* out, int M, int N, int K, int gated, void* stream) {
    if (M < 0 || N <= 0 || K <= 0 || N % 8 != 0 || K % 16 != 0)
        return fail(FRY_ERROR_SHAPE, "fry_int8_linear takes N a multiple of 8 and K a multiple of 16, got N " + std::to_string(N) +
                                         ", K " + std::to_string(K));
    if (!aligned16(x) || !aligned16(weight) || !aligned16(out) || (residual && !aligned16(residual)) || (original && !aligned16(original)))
        return fail(FRY_ERROR_SHAPE, "fry_int8_linear reads and writes 16-byte vectors: x, weight, out, residual and original must be 16-byte aligned");
    if (original && (!residual || !residual_scale || !input_scale))
        return fail(FRY_ERROR_SHAPE, "fry_int8_linear mixes the next input only with a residual and both scales");
    if (M == 0) return check(cudaSuccess, "");
    fry::GemmArgs args;
    args.x_scale = x_scale;
    args.w_scale = weight_scale;
    args.bias = bias;
    args.residual = residual;
    args.original = original;
    args.residual_scale = residual_scale;
    args.input_scale = input_scale;
    args.out = out;
    const int epilogue = gated ? fry::kEpiGated : residual == nullptr ? fry::kEpiBias : original == nullptr ? fry::kEpiResidual : fry::kEpiMix;
    std::string detail;
    return check(fry::gemm(0, epilogue, x, weight, args, M, N, K, as_stream(stream), &detail), "fry_int8_linear", detail);
}

int fry_int8_linear_normed(const uint16_t* x, const uint16_t* gain, float eps, const int8_t* weight, const float* weight_scale,
                           const uint16_t* bias, uint16_t* out, int M, int N, int K, int gated, void* stream) {
    if (M < 0 || N <= 0 || N % 8 != 0 || K != 768)
        return fail(FRY_ERROR_SHAPE, "fry_int8_linear_normed takes K = 768 and N a multiple of 8, got N " + std::to_string(N) + ", K " +
                                         std::to_string(K));
    if (!aligned16(x) || !aligned16(gain) || !aligned16(weight) || !aligned16(out))
        return fail(FRY_ERROR_SHAPE, "fry_int8_linear_normed reads and writes 16-byte vectors: x, gain, weight and out must be 16-byte aligned");
    if (M == 0) return check(cudaSuccess, "");
    fry::GemmArgs args;
    args.w_scale = weight_scale;
    args.bias = bias;
    args.out = out;
    args.norm_x = x;
    args.norm_gain = gain;
    args.norm_eps = eps;
    std::string detail;
    return check(fry::gemm(0, gated ? fry::kEpiGated : fry::kEpiBias, nullptr, weight, args, M, N, K, as_stream(stream), &detail),
                 "fry_int8_linear_normed", detail);
}

int fry_int8_matmul_i32(const int8_t* x, const int8_t* weight, int32_t* out, int M, int N, int K, void* stream) {
    if (M < 0 || N <= 0 || K <= 0 || N % 8 != 0 || K % 16 != 0)
        return fail(FRY_ERROR_SHAPE, "fry_int8_matmul_i32 takes N a multiple of 8 and K a multiple of 16");
    if (!aligned16(x) || !aligned16(weight) || !aligned16(out)) return fail(FRY_ERROR_SHAPE, "fry_int8_matmul_i32 needs 16-byte aligned tensors");
    if (M == 0) return check(cudaSuccess, "");
    fry::GemmArgs args;
    args.out = out;
    std::string detail;
    return check(fry::gemm(0, fry::kEpiInt32, x, weight, args, M, N, K, as_stream(stream), &detail), "fry_int8_matmul_i32", detail);
}

int fry_square_feature_rows(const int64_t* boards, int B, int32_t* rows, void* stream) {
    if (B < 0) return fail(FRY_ERROR_SHAPE, "fry_square_feature_rows needs B >= 0");
    if (!aligned16(boards) || (reinterpret_cast<uintptr_t>(rows) & 3u)) return fail(FRY_ERROR_SHAPE, "fry_square_feature_rows needs aligned tensors");
    return check(fry::square_feature_rows(boards, rows, B, as_stream(stream)), "fry_square_feature_rows");
}

int fry_int8_matmul_scaled_bf16(const int8_t* x, const float* x_scale, const int8_t* weight, const float* weight_scale, uint16_t* out, int M,
                                int N, int K, void* stream) {
    if (M < 0 || N <= 0 || K <= 0 || N % 8 != 0 || K % 16 != 0)
        return fail(FRY_ERROR_SHAPE, "fry_int8_matmul_scaled_bf16 takes N a multiple of 8 and K a multiple of 16, got N " + std::to_string(N) +
                                         ", K " + std::to_string(K));
    if (!aligned16(x) || !aligned16(weight) || !aligned16(out))
        return fail(FRY_ERROR_SHAPE, "fry_int8_matmul_scaled_bf16 needs 16-byte aligned x, weight and out");
    if (!x_scale || !weight_scale) return fail(FRY_ERROR_SHAPE, "fry_int8_matmul_scaled_bf16 needs both scales");
    if (M == 0) return check(cudaSuccess, "");
    fry::GemmArgs args;
    args.x_scale = x_scale;
    args.w_scale = weight_scale;
    args.out = out;
    std::string detail;
    return check(fry::gemm(0, fry::kEpiScaleBf16, x, weight, args, M, N, K, as_stream(stream), &detail), "fry_int8_matmul_scaled_bf16", detail);
}

int fry_attention_bf16(const uint16_t* q, const uint16_t* k, const uint16_t* v, uint16_t* out, int B, int heads, int seq, int head_dim,
                       void* stream) {
    if (B < 0 || seq != 64 || head_dim != 64 || heads <= 0 || heads > 1024 || B > 65535)
        return fail(FRY_ERROR_SHAPE, "fry_attention_bf16 takes sequences of 64 tokens with heads 64 wide (1 to 1024 heads, up to 65535 "
                                     "sequences), got seq " + std::to_string(seq) + ", head_dim " + std::to_string(head_dim));
    if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out))
        return fail(FRY_ERROR_SHAPE, "fry_attention_bf16 needs 16-byte aligned q, k, v and out");
    std::string detail;
    return check(fry::attention64(q, k, v, out, B, heads, as_stream(stream), &detail), "fry_attention_bf16", detail);
}

int fry_norm_quant(const uint16_t* x, const uint16_t* gain, float eps, int8_t* q, float* scale, int M, int D, void* stream) {
    if (M < 0 || D <= 0 || D % 8 != 0 || D > 1024) return fail(FRY_ERROR_SHAPE, "fry_norm_quant takes D a multiple of 8 up to 1024");
    if (!aligned16(x) || !aligned16(gain) || (reinterpret_cast<uintptr_t>(q) & 7u)) return fail(FRY_ERROR_SHAPE, "fry_norm_quant needs aligned rows");
    return check(fry::norm_quant(x, nullptr, nullptr, nullptr, gain, eps, nullptr, q, scale, M, D, as_stream(stream)), "fry_norm_quant");
}

int fry_mix_norm_quant(const uint16_t* x, const uint16_t* original, const uint16_t* residual_scale, const uint16_t* input_scale,
                       const uint16_t* gain, float eps, uint16_t* mixed, int8_t* q, float* scale, int M, int D, void* stream) {
    if (M < 0 || D <= 0 || D % 8 != 0 || D > 1024) return fail(FRY_ERROR_SHAPE, "fry_mix_norm_quant takes D a multiple of 8 up to 1024");
    if (!aligned16(x) || !aligned16(original) || !aligned16(mixed) || !aligned16(gain) || (reinterpret_cast<uintptr_t>(q) & 7u))
        return fail(FRY_ERROR_SHAPE, "fry_mix_norm_quant needs aligned rows");
    return check(fry::norm_quant(x, original, residual_scale, input_scale, gain, eps, mixed, q, scale, M, D, as_stream(stream)),
                 "fry_mix_norm_quant");
}

int fry_rotate_quant(const uint16_t* h, int8_t* q, float* scale, int M, int hidden, int width, void* stream) {
    if (M < 0 || hidden <= 0 || hidden % 8 != 0 || width % 32 != 0 || width > 1024 || hidden > width)
        return fail(FRY_ERROR_SHAPE, "fry_rotate_quant takes hidden a multiple of 8 and width a multiple of 32 up to 1024, width >= hidden");
    if (!aligned16(h) || !aligned16(q)) return fail(FRY_ERROR_SHAPE, "fry_rotate_quant needs 16-byte aligned rows");
    return check(fry::rotate_quant(h, q, scale, M, hidden, width, as_stream(stream)), "fry_rotate_quant");
}

int fry_pair_templates(const uint16_t* templates, uint16_t* paired, int templates_count, void* stream) {
    if (templates_count != 8) return fail(FRY_ERROR_SHAPE, "fry_pair_templates pairs 8 templates");
    if (!aligned16(paired)) return fail(FRY_ERROR_SHAPE, "fry_pair_templates needs a 16-byte aligned output");
    return check(fry::pair_templates(templates, paired, as_stream(stream)), "fry_pair_templates");
}

int fry_template_attention(const uint16_t* projected, const uint16_t* paired_templates, const uint16_t* q_gain, const uint16_t* k_gain,
                           uint16_t* out, int B, int heads, int kv_heads, int dq, int dv, int templates_count, float eps, void* stream) {
    if (B < 0) return fail(FRY_ERROR_SHAPE, "fry_template_attention takes B >= 0");
    if (!aligned16(projected) || !aligned16(out) || !aligned16(paired_templates))
        return fail(FRY_ERROR_SHAPE, "fry_template_attention needs 16-byte aligned projections, templates and outputs");
    std::string detail;
    return check(fry::template_attention(projected, paired_templates, q_gain, k_gain, out, B, heads, kv_heads, dq, dv, templates_count, eps,
                                         as_stream(stream), &detail),
                 "fry_template_attention", detail);
}

int fry_int8_linear_qk_norm(const int8_t* x, const float* x_scale, const int8_t* weight, const float* weight_scale, const uint16_t* bias,
                            const uint16_t* q_gain, const uint16_t* k_gain, float eps, uint16_t* out, int M, int N, int K, int heads,
                            int kv_heads, int dq, void* stream) {
    const int boundary = dq == 24 ? 48 : 16;
    if (M < 0 || N <= 0 || K <= 0 || N % 8 != 0 || K % 16 != 0 || (dq != 8 && dq != 16 && dq != 24) || heads <= 0 || kv_heads <= 0 ||
        (heads * dq) % boundary != 0 || ((heads + kv_heads) * dq) % boundary != 0 || (heads + kv_heads) * dq > N)
        return fail(FRY_ERROR_SHAPE, "fry_int8_linear_qk_norm takes query/key heads 8 or 16 wide whose blocks start on 16-column boundaries, "
                                     "or 24 wide on 48-column boundaries, within N (a multiple of 8), K a multiple of 16");
    if (!aligned16(x) || !aligned16(weight) || !aligned16(out)) return fail(FRY_ERROR_SHAPE, "fry_int8_linear_qk_norm needs 16-byte aligned x, weight and out");
    if (!x_scale || !weight_scale || !q_gain || !k_gain) return fail(FRY_ERROR_SHAPE, "fry_int8_linear_qk_norm needs both scales and both gains");
    if (M == 0) return check(cudaSuccess, "");
    fry::GemmArgs args;
    args.x_scale = x_scale;
    args.w_scale = weight_scale;
    args.bias = bias;
    args.out = out;
    args.q_gain = q_gain;
    args.k_gain = k_gain;
    args.qk_dq = dq;
    args.qk_queries = heads * dq;
    args.qk_keys = (heads + kv_heads) * dq;
    args.norm_eps = eps;
    std::string detail;
    return check(fry::gemm(0, fry::kEpiBiasQkNorm, x, weight, args, M, N, K, as_stream(stream), &detail), "fry_int8_linear_qk_norm", detail);
}

int fry_template_attention_normed(const uint16_t* projected, const uint16_t* paired_templates, uint16_t* out, int B, int heads, int kv_heads,
                                  int dq, int dv, int templates_count, void* stream) {
    if (B < 0) return fail(FRY_ERROR_SHAPE, "fry_template_attention_normed takes B >= 0");
    if (dq != 8 && dq != 16 && dq != 24) return fail(FRY_ERROR_SHAPE, "fry_template_attention_normed takes dq 8, 16 or 24");
    if (!aligned16(projected) || !aligned16(out) || !aligned16(paired_templates))
        return fail(FRY_ERROR_SHAPE, "fry_template_attention_normed needs 16-byte aligned projections, templates and outputs");
    std::string detail;
    return check(fry::template_attention(projected, paired_templates, nullptr, nullptr, out, B, heads, kv_heads, dq, dv, templates_count, 0.0f,
                                         as_stream(stream), &detail, true),
                 "fry_template_attention_normed", detail);
}

int fry_linear(const uint16_t* x, const uint16_t* weight, const void* bias, const uint16_t* residual, void* out, int M, int N, int K,
               int out_fp32, void* stream) {
    if (M < 0 || N <= 0 || K <= 0 || N % 8 != 0 || K % 8 != 0)
        return fail(FRY_ERROR_SHAPE, "fry_linear takes N and K multiples of 8");
    if (out_fp32 && residual) return fail(FRY_ERROR_SHAPE, "fry_linear adds no residual to an fp32 output");
    if (!aligned16(x) || !aligned16(weight) || !aligned16(out) || (residual && !aligned16(residual)))
        return fail(FRY_ERROR_SHAPE, "fry_linear needs 16-byte aligned tensors");
    if (M == 0) return check(cudaSuccess, "");
    fry::GemmArgs args;
    if (out_fp32)
        args.bias_f32 = static_cast<const float*>(bias);
    else
        args.bias = static_cast<const uint16_t*>(bias);
    args.residual = residual;
    args.out = out;
    std::string detail;
    return check(fry::gemm(1, out_fp32 ? fry::kEpiLinearF32 : fry::kEpiLinearF16, x, weight, args, M, N, K, as_stream(stream), &detail),
                 "fry_linear", detail);
}

int fry_linear_full(const uint16_t* x, const uint16_t* weight, const uint16_t* bias, const uint16_t* residual, const uint16_t* original,
                    const uint16_t* residual_scale, const uint16_t* input_scale, uint16_t* out, int M, int N, int K, int gated, void* stream) {
    if (M < 0 || N <= 0 || K <= 0 || N % 8 != 0 || K % 8 != 0) return fail(FRY_ERROR_SHAPE, "fry_linear_full takes N and K multiples of 8");
    if (gated && (residual || original)) return fail(FRY_ERROR_SHAPE, "fry_linear_full's gated form adds no residual and mixes no input");
    if (original && (!residual || !residual_scale || !input_scale))
        return fail(FRY_ERROR_SHAPE, "fry_linear_full mixes the next input only with a residual and both scales");
    if (!aligned16(x) || !aligned16(weight) || !aligned16(out) || (residual && !aligned16(residual)) || (original && !aligned16(original)))
        return fail(FRY_ERROR_SHAPE, "fry_linear_full needs 16-byte aligned tensors");
    if (M == 0) return check(cudaSuccess, "");
    fry::GemmArgs args;
    args.bias = bias;
    args.residual = residual;
    args.original = original;
    args.residual_scale = residual_scale;
    args.input_scale = input_scale;
    args.out = out;
    const int epilogue = gated ? fry::kEpiGatedF16 : original ? fry::kEpiMixF16 : fry::kEpiLinearF16;
    std::string detail;
    return check(fry::gemm(1, epilogue, x, weight, args, M, N, K, as_stream(stream), &detail), "fry_linear_full", detail);
}

int fry_linear_norm_quant(const uint16_t* x, const uint16_t* weight, const uint16_t* bias, const uint16_t* residual, uint16_t* out,
                          const uint16_t* gain, float eps, int8_t* q, float* scale, int M, int N, int K, void* stream) {
    if (M < 0 || N <= 0 || K <= 0 || N % 256 != 0 || N > 1024 || K % 8 != 0)
        return fail(FRY_ERROR_SHAPE, "fry_linear_norm_quant takes N a multiple of 256 up to 1024 and K a multiple of 8, got N " +
                                         std::to_string(N) + ", K " + std::to_string(K));
    if (!aligned16(x) || !aligned16(weight) || !aligned16(out) || !aligned16(gain) || !aligned16(q) || !scale || (residual && !aligned16(residual)))
        return fail(FRY_ERROR_SHAPE, "fry_linear_norm_quant needs 16-byte aligned tensors and a scale output");
    if (M == 0) return check(cudaSuccess, "");
    fry::GemmArgs args;
    args.bias = bias;
    args.residual = residual;
    args.out = out;
    args.norm_gain = gain;
    args.norm_eps = eps;
    args.norm_q = q;
    args.norm_scale = scale;
    std::string detail;
    return check(fry::gemm(1, fry::kEpiLinearNorm, x, weight, args, M, N, K, as_stream(stream), &detail), "fry_linear_norm_quant", detail);
}

int fry_board_embedding(const int64_t* boards, const uint16_t* embed, const uint16_t* position, const uint16_t* table, uint16_t* out,
                        int B, int D, void* stream) {
    if (B < 0 || D <= 0 || D % 8 != 0) return fail(FRY_ERROR_SHAPE, "fry_board_embedding takes D a multiple of 8");
    if (!aligned16(embed) || !aligned16(position) || !aligned16(table) || !aligned16(out))
        return fail(FRY_ERROR_SHAPE, "fry_board_embedding needs 16-byte aligned tables and output");
    return check(fry::board_embedding(boards, embed, position, table, out, B, D, as_stream(stream)), "fry_board_embedding");
}

size_t fry_heads_workspace_bytes(int B, int D) { return B > 0 && D > 0 ? fry::heads_workspace_bytes(B, D) : 0; }

int fry_heads(const uint16_t* stream_x, const FryHeads* heads, float eps, float* rows, void* workspace, size_t workspace_bytes, int B,
              int D, void* stream) {
    if (!heads || B < 0) return fail(FRY_ERROR_SHAPE, "fry_heads needs its weights and B >= 0");
    if (D < 16 || D % 16 != 0 || D > 1024) return fail(FRY_ERROR_SHAPE, "fry_heads takes d_model a multiple of 16 from 16 to 1024, got " + std::to_string(D));
    if (!aligned16(stream_x) || !aligned16(workspace) || !aligned16(heads->a_weight) || !aligned16(heads->ln_gain))
        return fail(FRY_ERROR_SHAPE, "fry_heads needs 16-byte aligned tensors");
    fry::HeadWeights w{heads->ln_gain,     heads->a_weight,    heads->a_bias,     heads->narrow_weight, heads->narrow_bias,
                       heads->hidden_weight, heads->hidden_bias, heads->out_weight, heads->out_bias,      heads->bins};
    std::string detail;
    return check(fry::heads(stream_x, w, eps, rows, workspace, workspace_bytes, B, D, as_stream(stream), &detail), "fry_heads", detail);
}

size_t fry_forward_workspace_bytes(const FryNetwork* n, int B) {
    if (!n || B <= 0) return 0;
    const size_t M = static_cast<size_t>(B) * 70, D = n->d_model;
    int widest = 0;
    for (int i = 0; i < n->layers; ++i) {
        const int rows = projection_rows(n, n->blocks[i].dq);
        widest = rows > widest ? rows : widest;
    }
    const size_t q_width = D > static_cast<size_t>(n->down_width) ? D : static_cast<size_t>(n->down_width);
    return round_up(M * D * 2) * 3 + round_up(M * q_width) + round_up(M * 4) + round_up(M * widest * 2) + round_up(M * n->hidden * 2) +
           round_up(fry::heads_workspace_bytes(B, n->d_model));
}

int fry_forward(const FryNetwork* n, const int64_t* boards, int B, float* rows, void* workspace, size_t workspace_bytes, void* stream) {
    return run_forward(n, boards, nullptr, B, rows, nullptr, workspace, workspace_bytes, stream);
}

size_t fry_forward_lean_workspace_bytes(const FryNetwork* n, int B) {
    if (!n || B <= 0) return 0;
    return fry_forward_workspace_bytes(n, B) + round_up(static_cast<size_t>(B) * (kAnswerWidth * 4));
}

int fry_forward_lean(const FryNetwork* n, const uint8_t* lean_rows, int B, float* answers, void* workspace, size_t workspace_bytes,
                     void* stream) {
    if (!n || B < 0) return fail(FRY_ERROR_SHAPE, "fry_forward_lean needs a network and B >= 0");
    if (B == 0) return check(cudaSuccess, "");
    if (workspace_bytes < fry_forward_lean_workspace_bytes(n, B))
        return fail(FRY_ERROR_SHAPE, "fry_forward_lean's workspace is smaller than fry_forward_lean_workspace_bytes");
    if (!lean_rows || !answers || !aligned16(workspace)) return fail(FRY_ERROR_SHAPE, "fry_forward_lean needs its rows, answers and a 16-byte aligned workspace");
    // the whole answer rows sit at the end of the workspace, the forward's own scratch before them
    const size_t forward_bytes = fry_forward_workspace_bytes(n, B);
    float* rows = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + forward_bytes);
    return run_forward(n, nullptr, lean_rows, B, rows, answers, workspace, forward_bytes, stream);
}

size_t fry_gptq_workspace_bytes(int N, int K) { return N > 0 && K > 0 ? fry::GptqWorkspace(N, K).total : 0; }

int fry_gptq(const double* weight, const double* hessian, int N, int K, int8_t* q, float* scale, void* workspace,
             size_t workspace_bytes, void* stream) {
    if (!weight || !hessian || !q || !scale || !workspace)
        return fail(FRY_ERROR_SHAPE, "fry_gptq needs its weight, hessian, outputs and workspace");
    if (!aligned16(workspace) || reinterpret_cast<uintptr_t>(weight) % 8 != 0 || reinterpret_cast<uintptr_t>(hessian) % 8 != 0)
        return fail(FRY_ERROR_SHAPE, "fry_gptq needs fp64-aligned inputs and a 16-byte aligned workspace");
    std::string detail;
    const cudaError_t status = fry::gptq(weight, hessian, N, K, q, scale, workspace, workspace_bytes, as_stream(stream), &detail);
    if (status == cudaErrorInvalidValue && !detail.empty()) return fail(FRY_ERROR_SHAPE, detail);
    return check(status, "fry_gptq");
}

int fry_hessian_accumulate(const double* x, int rows, int K, double* hessian, void* stream) {
    if ((rows > 0 && !x) || !hessian || reinterpret_cast<uintptr_t>(x) % 8 != 0 || reinterpret_cast<uintptr_t>(hessian) % 8 != 0)
        return fail(FRY_ERROR_SHAPE, "fry_hessian_accumulate needs fp64-aligned x and hessian");
    std::string detail;
    const cudaError_t status = fry::hessian_accumulate(x, rows, K, hessian, as_stream(stream), &detail);
    if (status == cudaErrorInvalidValue && !detail.empty()) return fail(FRY_ERROR_SHAPE, detail);
    return check(status, "fry_hessian_accumulate");
}

}  // extern "C"
