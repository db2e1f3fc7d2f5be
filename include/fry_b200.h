/* fry_b200: the C ABI of the B200 (sm_100a) int8 inference engine for Fry's network (GilliamWong/chess-transformer).
 *
 * Every pointer argument is a device pointer unless stated otherwise; fp16 tensors are passed as uint16_t bit patterns;
 * every array is dense row-major. `stream` is a cudaStream_t (NULL: the legacy default stream). The block ops, the heads,
 * the forward and GPTQ only enqueue work: they do not synchronise the stream, allocate device memory or keep a pointer
 * between calls (the caller provides the scratch that the *_workspace_bytes functions size), so the block ops, the heads
 * and the forward can be recorded into CUDA graphs, as GraphedBatches and the lanes record the forward. The lanes
 * (fry_lanes_*) own their memory, streams and graphs, and fry_lanes_create, _collect and _settle wait on the GPU; so
 * does fry_device_status. Each returns 0 on success or a nonzero code; fry_last_error() gives the calling thread's last
 * message. Shapes a kernel does not take are refused on the host with FRY_ERROR_SHAPE before anything is
 * enqueued (the reference raises ValueError for these, model/int8_blocks.py:111-112, model/fused_blocks.py:116-117).
 *
 * Faults the kernels can detect (a wait that timed out, a board token outside the vocabulary) are recorded in a device
 * status word that fry_device_status() reads; the kernels never trap.
 */
#ifndef FRY_B200_H
#define FRY_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FRY_OK 0
#define FRY_ERROR_SHAPE 1   /* a shape or alignment the kernels do not take */
#define FRY_ERROR_CUDA 2    /* a CUDA runtime or driver call failed */

/* The calling thread's last error message ("" after a success). The string stays valid until the thread's next call
 * into the library: read it after the call that failed, not in the same expression. */
const char* fry_last_error(void);

/* The library version string. */
const char* fry_version(void);

/* Reads the current device's status word: *code 0 if no kernel recorded a fault, else the code (1 a bounded wait timed
 * out, 2 a board token outside the vocabulary, 3 a launch shape a kernel does not take, 4 misaligned shared memory, 5 a
 * lean lane's answer column outside the answer row, 6 a GPTQ Hessian that is not positive definite) and *where its
 * site. clear != 0 resets it. Synchronous. */
int fry_device_status(int* code, int* where, int clear);

/* Every wait of a kernel on a barrier (a TMA load, a tensor-core commit, a cluster peer) is bounded: after the current
 * device's wait limit, 2 s unless set here, it records code 1 in the status word (where = the wait's site) and the
 * kernel returns without touching what it waited for, so a stalled kernel ends and the context stays usable. The limit
 * is per device (the current one), 1 us to 60 s; kernels already running keep the limit they read. Synchronous.
 * The reference's counterpart is its host-side fallback on a failing kernel (model/int8_cuda.py:370-381). */
int fry_set_wait_limit_ns(uint64_t limit_ns);
int fry_wait_limit_ns(uint64_t* limit_ns);

/* A health check of that path: enqueues one kernel whose thread waits on a barrier that nothing arrives at, so the wait
 * runs out after the limit and the status word reads code 1, where 90. No reference counterpart. */
int fry_wait_probe(void* stream);

/* ---- block ops: each replaces one torch custom op of the reference ----------------------------------------------- */

/* `chess::int8_linear` (model/int8_blocks.py:132-139, kernels :66-128 and model/int8_cuda.py:34-183):
 * out[M, N] fp16 = epilogue(x[M, K] int8 . weight^T), weight int8 [N, K] ([2N, K], gate rows then up rows, if gated).
 * The epilogue is picked as the reference picks it (model/int8_cuda.py:163-178):
 *   gated                      fp16((g * sigmoid(g)) * u), g and u = (acc * x_scale) * weight_scale
 *   residual == NULL           fp16(fma(acc * x_scale, weight_scale, bias))        (bias may be NULL: zero)
 *   residual, original NULL    fp16(fma(acc * x_scale, weight_scale, residual))
 *   residual and original      the above rounded to fp16, then fp16(fma(stream, *residual_scale, original * *input_scale))
 * x_scale fp32 [M], weight_scale fp32 [N] ([2N] gated); out may alias residual. N must be a multiple of 8, K of 16. */
int fry_int8_linear(const int8_t* x, const float* x_scale, const int8_t* weight, const float* weight_scale, const uint16_t* bias,
                    const uint16_t* residual, const uint16_t* original, const uint16_t* residual_scale, const uint16_t* input_scale,
                    uint16_t* out, int M, int N, int K, int gated, void* stream);

/* `chess::norm_quant` feeding `chess::int8_linear` as one kernel: out = int8_linear(norm_quant(x, gain, eps)) with the
 * bias (gated == 0; bias may be NULL) or the gated epilogue, the pair `Int8Block.forward` runs for ln1 -> projection and
 * ln2 -> gate_up (model/int8_blocks.py:274-288; ops :191-193 and :132-139). The int8 rows and their scales are made in
 * the GEMM's prologue and stay in shared memory; the bits equal those of fry_norm_quant then fry_int8_linear.
 * x fp16 [M, K] and gain fp16 [K], 16-byte aligned; K must be 768 (the model width), N a multiple of 8. */
int fry_int8_linear_normed(const uint16_t* x, const uint16_t* gain, float eps, const int8_t* weight, const float* weight_scale,
                           const uint16_t* bias, uint16_t* out, int M, int N, int K, int gated, void* stream);

/* The int32 sums x[M, K] . weight[N, K]^T of the same tensor-core kernel, for bit-exact checks. No reference
 * counterpart exposes them; they are the `acc` of model/int8_blocks.py:85-92. */
int fry_int8_matmul_i32(const int8_t* x, const int8_t* weight, int32_t* out, int M, int N, int K, void* stream);

/* The benchmark's isolated int8 GEMM: out[M, N] bf16 = bf16((acc * x_scale[m]) * weight_scale[n]), acc = x[M, K] .
 * weight[N, K]^T in int32, on the same tensor-core kernel as fry_int8_linear. No reference op outputs bf16; the
 * reference's own int8 linear with no bias is fp16(fma(acc * x_scale, weight_scale, 0)) (model/int8_cuda.py:163-165).
 * N a multiple of 8, K of 16; x, weight and out 16-byte aligned. */
int fry_int8_matmul_scaled_bf16(const int8_t* x, const float* x_scale, const int8_t* weight, const float* weight_scale, uint16_t* out, int M,
                                int N, int K, void* stream);

/* The benchmark's isolated attention: out = softmax(q k^T / sqrt(64)) v per sequence and head, bf16 in and out, fp32
 * sums and softmax. q, k, v and out are [B, seq, heads * head_dim] (a projection's rows, heads side by side). Takes
 * seq 64 and head_dim 64 only, 1 to 1024 heads, B up to 65535. The reference's attention of this shape family is its
 * template attention (model/fused_blocks.py:54-97), which fry_template_attention replaces; this one has no bias, no
 * norms and no grouped heads. */
int fry_attention_bf16(const uint16_t* q, const uint16_t* k, const uint16_t* v, uint16_t* out, int B, int heads, int seq, int head_dim,
                       void* stream);

/* `chess::norm_quant` (model/int8_blocks.py:191-193, kernel :156-175): q[M, D] int8, scale[M] fp32 of
 * RMSNorm(x) * gain, a row's scale its absmax / 127. D a multiple of 8 up to 1024. */
int fry_norm_quant(const uint16_t* x, const uint16_t* gain, float eps, int8_t* q, float* scale, int M, int D, void* stream);

/* `chess::mix_norm_quant` (model/int8_blocks.py:201-207): mixed = fp16(*residual_scale * x + *input_scale * original),
 * then norm_quant of mixed. */
int fry_mix_norm_quant(const uint16_t* x, const uint16_t* original, const uint16_t* residual_scale, const uint16_t* input_scale,
                       const uint16_t* gain, float eps, uint16_t* mixed, int8_t* q, float* scale, int M, int D, void* stream);

/* `chess::rotate_quant` (model/int8_blocks.py:234-246, kernel :216-231): h[M, hidden] fp16 zero-padded to width, times the
 * block-diagonal 32x32 Sylvester Hadamard matrix (the reference's hadamard_signs, model/int8_blocks.py:54-58, built in),
 * then int8 rows q[M, width] and scale[M]. width a multiple of 32 up to 1024, hidden a multiple of 8. */
int fry_rotate_quant(const uint16_t* h, int8_t* q, float* scale, int M, int hidden, int width, void* stream);

/* `paired_templates` (model/attention_cuda.py:412-434): the position templates fp16 [8, 64, 64] re-laid as
 * paired [64, 64, 8] (paired[i][j][t] = templates[t][i][j]), the operand fry_template_attention reads. Run it once per
 * set of templates (the reference caches its pairing per tensor). */
int fry_pair_templates(const uint16_t* templates, uint16_t* paired, int templates_count, void* stream);

/* `chess::template_attention` (model/fused_blocks.py:104-171; model/attention_cuda.py:444-461): projected [B, 70, W] fp16
 * with W = heads*dq + kv_heads*dq + kv_heads*dv + heads*templates_count (q | k | v | template mix), paired_templates from
 * fry_pair_templates, q_gain and k_gain fp16 [dq] -> out [B, 70, heads*dv] fp16. Takes dv 32, 8 templates, dq a multiple
 * of 8 up to 32, heads/kv_heads groups that fit 8 query heads a CTA. */
int fry_template_attention(const uint16_t* projected, const uint16_t* paired_templates, const uint16_t* q_gain, const uint16_t* k_gain,
                           uint16_t* out, int B, int heads, int kv_heads, int dq, int dv, int templates_count, float eps, void* stream);

/* `chess::int8_linear` for the projection (model/int8_blocks.py:132-139, bias epilogue) with the next op's q and k
 * RMSNorm (`template_attention`'s q_norm and k_norm with their gains, model/fused_blocks.py:54-97) in its epilogue:
 * out[M, N] fp16 is fry_int8_linear's output with columns [0, heads*dq) (queries) and [heads*dq, (heads+kv_heads)*dq)
 * (keys) replaced, head by head, by fp16((x * inverse) * gain), inverse = rsqrt(mean(x^2) + eps), summed in the order
 * fry_template_attention sums them, so fry_template_attention_normed on it equals fry_template_attention on the plain
 * projection bit for bit. dq 8 or 16 with the query and key blocks on 16-column boundaries, or dq 24 with them on
 * 48-column boundaries (heads * 24 and (heads + kv_heads) * 24 multiples of 48). */
int fry_int8_linear_qk_norm(const int8_t* x, const float* x_scale, const int8_t* weight, const float* weight_scale, const uint16_t* bias,
                            const uint16_t* q_gain, const uint16_t* k_gain, float eps, uint16_t* out, int M, int N, int K, int heads,
                            int kv_heads, int dq, void* stream);

/* fry_template_attention on a projection whose query and key columns fry_int8_linear_qk_norm has normalised: the
 * queries and keys are used as they are. dq 8, 16 or 24; otherwise as fry_template_attention. */
int fry_template_attention_normed(const uint16_t* projected, const uint16_t* paired_templates, uint16_t* out, int B, int heads, int kv_heads,
                                  int dq, int dv, int templates_count, void* stream);

/* `chess::linear` (model/fused_blocks.py:308-313, kernel :229-304) for fp16 inputs: out[M, N] = (x[M, K] . weight^T + bias)
 * + residual, fp32 accumulation, fp16 out (out_fp32 == 0) or fp32 out without residual (out_fp32 != 0, the reference's
 * accumulate_fp32). weight is [N, K] fp16 (the reference stores it transposed, [K, N]). bias fp16 [N] (fp32 [N] when
 * out_fp32) and residual [M, N] may be NULL; out may alias residual. N a multiple of 8, K of 8. */
int fry_linear(const uint16_t* x, const uint16_t* weight, const void* bias, const uint16_t* residual, void* out, int M, int N, int K,
               int out_fp32, void* stream);

/* `chess::linear` (model/fused_blocks.py:308-313, epilogue :209-225) with every fp16 form the fp16 blocks use:
 * out[M, N] fp16 from fp32 sums acc = x . weight^T, then gated != 0: fp16((g * sigmoid(g)) * u), g = acc + bias over
 * weight rows [0, N), u over rows [N, 2N) (weight [2N, K]); else (acc + bias) + residual, and with original (and both
 * scales) the sum rounded to fp16 then fp16(fma(stream, *residual_scale, original * *input_scale)). bias, residual and
 * original may be NULL (original needs residual); out may alias residual. N a multiple of 8, K of 8. */
int fry_linear_full(const uint16_t* x, const uint16_t* weight, const uint16_t* bias, const uint16_t* residual, const uint16_t* original,
                    const uint16_t* residual_scale, const uint16_t* input_scale, uint16_t* out, int M, int N, int K, int gated, void* stream);

/* `chess::linear` (fp16, as fry_linear) feeding `chess::norm_quant` (model/int8_blocks.py:191-193) in one kernel, the pair
 * `Int8Block.forward` runs for attention-out -> ln2 (model/int8_blocks.py:274-288): out[M, N] fp16 = (x . weight^T + bias)
 * + residual, then q[M, N] int8 and scale[M] fp32 of RMSNorm(out) * gain. The N / 256 CTAs that share a 128-row block
 * form a thread-block cluster and sum each row's squares through distributed shared memory. out equals fry_linear's bit
 * for bit; q and scale equal fry_norm_quant's to within its rounding: the squares are summed in another order, and the
 * row's absmax is taken as inverse * max|out * gain| (within fp32 rounding of max|(out * inverse) * gain|).
 * N a multiple of 256 up to 1024, K of 8; x, weight, out, residual, gain and q 16-byte aligned; out may alias residual. */
int fry_linear_norm_quant(const uint16_t* x, const uint16_t* weight, const uint16_t* bias, const uint16_t* residual, uint16_t* out,
                          const uint16_t* gain, float eps, int8_t* q, float* scale, int M, int N, int K, void* stream);

/* `chess::board_embedding` / `chess::input_embedding` (model/fused_blocks.py:397-406,495-507, SquareFeatures.indices
 * model/model.py:147-169): boards int64 [B, 70] -> out [B, 70, D] fp16 = embed[token] + position[t] + fp16(sum of the 23
 * square-feature rows of table). embed [81, D], position [70, D], table [1735, D] fp16. A token outside the vocabulary
 * (0..12 on squares, 0..80 on the metadata) is read as 0 and recorded in the device status word. */
int fry_board_embedding(const int64_t* boards, const uint16_t* embed, const uint16_t* position, const uint16_t* table, uint16_t* out,
                        int B, int D, void* stream);

/* `SquareFeatures.indices` (model/model.py:134-169) with each feature's first row added: boards int64 [B, 70] -> rows
 * int32 [B, 64, 23], the row of the square-feature table each square reads for each of the 23 features (the rows
 * fry_board_embedding sums). For offline work on the checkpoint's own precision, such as calibration. */
int fry_square_feature_rows(const int64_t* boards, int B, int32_t* rows, void* stream);

/* The heads after the last block, as the reference runs them on B200 (model/fused_blocks.py:863-874, weights folded by
 * head_weights :815-824) with answer_rows (engine/inference.py:19-23). stream [B, 70, D] fp16 -> rows [B, 1969] fp32.
 * workspace: device scratch of fry_heads_workspace_bytes(B, D) bytes. */
typedef struct FryHeads {
    const uint16_t* ln_gain;       /* fp16 [D], the final RMSNorm's gain */
    const uint16_t* a_weight;      /* fp16 [D, D]: (W_f^T W_t / sqrt D)^T, row n = output column n */
    const float* a_bias;           /* fp32 [D]: W_t^T b_f / sqrt D */
    const float* narrow_weight;    /* fp32 [21, D]: (b_t W_f)/sqrt D, promotion_projection, board_down_project */
    const float* narrow_bias;      /* fp32 [21] */
    const float* hidden_weight;    /* fp32 [D, 1120]: eval_head[0] */
    const float* hidden_bias;      /* fp32 [D] */
    const float* out_weight;       /* fp32 [bins, D]: eval_head[2] */
    const float* out_bias;         /* fp32 [bins] */
    int bins;
} FryHeads;

size_t fry_heads_workspace_bytes(int B, int D);
int fry_heads(const uint16_t* stream_x, const FryHeads* heads, float eps, float* rows, void* workspace, size_t workspace_bytes, int B,
              int D, void* stream);

/* fry_heads without a workspace, for callers that cannot allocate device memory when they evaluate positions (a
 * thread in the middle of a stream capture, where cudaMalloc is not allowed; a latency-bound search loop that must not
 * risk the device-wide synchronisation an allocation can cause; a host in another language with no device allocator).
 * No counterpart in the reference: its heads always allocate through torch.
 * The scratch is a fixed array inside the library (about 5.5 MiB, held by every GPU that loads the library until
 * exit), so a call takes at most FRY_HEADS_NOALLOC_MAX_BOARDS boards of d_model up to FRY_HEADS_NOALLOC_MAX_D_MODEL;
 * larger calls return FRY_ERROR_SHAPE before anything is enqueued. All calls on a device share the array, which keeps
 * the last call's contents: calls whose work overlaps on the GPU race and must be ordered by the caller. The first call
 * on a device (and the first after a device reset) looks up the array's device address; make it before any stream
 * capture on that device. d_model must be a multiple of 16 from 16. */
#define FRY_HEADS_NOALLOC_MAX_BOARDS 16
#define FRY_HEADS_NOALLOC_MAX_D_MODEL 768
int fry_heads_noalloc(const uint16_t* stream_x, const FryHeads* heads, float eps, float* rows, int B, int D, void* stream);

/* ---- the whole forward ------------------------------------------------------------------------------------------- */

/* One block: an int8 block as `Int8Block` holds it (model/int8_blocks.py:254-272) with the layout of
 * engine/quantization.py:129-139, or (precision FRY_BLOCK_FP16) an fp16 block as `FusedBlock` runs it
 * (model/fused_blocks.py:325-354), whose projection, gate_up and down are fp16 in nn.Linear's [out, in] layout, the down
 * [D, hidden] times the stream's 1/16, and whose scales are unused. */
#define FRY_BLOCK_INT8 0
#define FRY_BLOCK_FP16 1
typedef struct FryBlock {
    int dq;
    const uint16_t* ln1;                 /* fp16 [D] */
    const uint16_t* ln2;                 /* fp16 [D] */
    const uint16_t* residual_scale;      /* fp16 [1] */
    const uint16_t* input_scale;         /* fp16 [1] */
    const uint16_t* q_gain;              /* fp16 [dq] */
    const uint16_t* k_gain;              /* fp16 [dq] */
    const void* projection;              /* int8 (fp16) [36*dq + 576 (generally heads*dq + kv*dq + kv*dv + heads*templates), D] */
    const float* projection_scale;       /* fp32 [rows of projection] */
    const uint16_t* projection_bias;     /* fp16 [rows of projection] */
    const uint16_t* combine_heads;       /* fp16 [D, D], row n = output column n (the reference's [K, N] transposed) */
    const uint16_t* combine_heads_bias;  /* fp16 [D] */
    const void* gate_up;                 /* int8 (fp16) [2*hidden, D], gate rows then up rows */
    const float* gate_up_scale;          /* fp32 [2*hidden] */
    const void* down;                    /* int8 [D, width], padded and Hadamard-rotated (fp16 [D, hidden]) */
    const float* down_scale;             /* fp32 [D], times the stream's 1/16 */
    int precision;                       /* FRY_BLOCK_INT8 or FRY_BLOCK_FP16 */
} FryBlock;

/* The network: FusedTransformer with its blocks int8 (Int8Block) or fp16 (FusedBlock) (model/fused_blocks.py:829-878,
 * model/int8_blocks.py:292-298), a down mixing the next block's input when both are of one precision, a block after one
 * of the other precision mixing its own (link_input_mixes, model/fused_blocks.py:358-363).
 * This struct and the blocks array live in host memory; every tensor pointer in them is a device pointer. */
typedef struct FryNetwork {
    int d_model, layers, heads, kv_heads, dv, templates_count, hidden, down_width;
    float eps;
    const uint16_t* embed;      /* fp16 [81, D], times 1/16 */
    const uint16_t* position;   /* fp16 [70, D], times 1/16 */
    const uint16_t* table;      /* fp16 [1735, D], times 1/16 */
    const uint16_t* templates;  /* fp16 [64, 64, 8]: the position templates paired by fry_pair_templates */
    const FryBlock* blocks;     /* [layers], host memory */
    FryHeads head_weights;      /* the heads' weights */
} FryNetwork;

/* Device scratch the forward needs for B boards. */
size_t fry_forward_workspace_bytes(const FryNetwork* network, int B);

/* `FusedTransformer.forward` + `answer_rows` (model/fused_blocks.py:856-862, engine/inference.py:19-23): boards int64
 * [B, 70] -> rows fp32 [B, 1969] (1968 move logits, then the expected score). */
int fry_forward(const FryNetwork* network, const int64_t* boards, int B, float* rows, void* workspace, size_t workspace_bytes,
                void* stream);

/* The forward on lean lanes (engine/inference.py:94-100,130-135, the Rust round loop's wire format): lean_rows uint8
 * [B, 508], a board's 70 token bytes then 219 int16 (little-endian) answer columns, the legal moves' and, after them,
 * 1968, the expected score's (engine/selfplay_rs/src/lib.rs:330-333) -> answers fp32 [B, 219], the columns of the board's
 * answer row, gathered by the heads' last kernel. A column outside [0, 1968] answers 0 and sets the device status
 * (code 5, where = the board). The workspace holds the forward's scratch and the whole rows. */
size_t fry_forward_lean_workspace_bytes(const FryNetwork* network, int B);
int fry_forward_lean(const FryNetwork* network, const uint8_t* lean_rows, int B, float* answers, void* workspace, size_t workspace_bytes,
                     void* stream);

/* ---- GPTQ: the offline rounding of a block's weights to Int8Weights ---------------------------------------------------
 * `gptq` (engine/quantization.py:76-99, Frantar et al. 2022) in fp64: weight [N, K] and the input Hessian [K, K] (both
 * fp64, device) -> q int8 [N, K] and scale fp32 [N], as the reference returns them. Inputs whose Hessian diagonal is zero
 * get zero weights; the diagonal is dampened by 0.01 of its mean; columns are rounded half to even in blocks of 128,
 * each column's error spread over the later ones through the inverse Hessian's upper Cholesky factor. A Hessian that is
 * not positive definite is recorded in the device status (code 6, where = the column), as the reference's
 * torch.linalg.cholesky raises. Enqueue only; 0 < N <= 262144, 0 < K <= 4096. */
size_t fry_gptq_workspace_bytes(int N, int K);
int fry_gptq(const double* weight, const double* hessian, int N, int K, int8_t* q, float* scale, void* workspace,
             size_t workspace_bytes, void* stream);
/* The Hessians GPTQ takes (`input_hessians`, engine/quantization.py:103-119): hessian [K, K] += x^T x for a matmul's
 * inputs x [rows, K], fp64 on the device. The sum is exactly symmetric. Enqueue only; 0 < K <= 4096. */
int fry_hessian_accumulate(const double* x, int rows, int K, double* hessian, void* stream);

/* ---- lanes: the batch runtime in C++ ------------------------------------------------------------------------------
 * `GraphedBatches` and `Lane` (engine/inference.py:85-225) with the CUDA runtime calls of engine/cuda_runtime.py, and no
 * Python between batches. A FryLanes holds `in_flight` lanes on the device current at creation. Each lane has its own
 * stream, one CUDA graph of the forward per batch size in `sizes` (ascending), pinned host buffers for the boards in and
 * the answers out, and a done event. fry_lanes_launch copies a batch's boards in, replays the smallest graph that holds
 * it and returns; fry_lanes_collect copies its answers out and waits for them. At most one batch is out a lane.
 * A lean FryLanes (lean != 0) takes rows of FRY_LEAN_ROW bytes (70 token bytes, then FRY_LEAN_COLUMNS int16 answer
 * columns) and answers FRY_LEAN_COLUMNS floats a board, as fry_forward_lean; otherwise it takes boards int64 [n, 70]
 * and answers rows fp32 [n, 1969], as fry_forward. The graphs read the network's weights where they were at
 * fry_lanes_create: keep them in place while the FryLanes lives. A call out of order (a launch on a lane whose batch is
 * out, a collect of a lane with none, no free lane) returns FRY_ERROR_STATE, as the reference raises RuntimeError. */
#define FRY_ERROR_STATE 3   /* a lane call out of order */
#define FRY_LEAN_ROW 508
#define FRY_LEAN_COLUMNS 219
typedef struct FryLanes FryLanes;

/* The raw handles of a lane, as `Lane.handles()` gives them (engine/inference.py:138-142): every size's graph writes
 * the lane's one answers buffer. Pointers are host-pinned (`*_host`) or device memory. */
typedef struct FryLaneHandles {
    int device;
    void* stream;        /* cudaStream_t */
    void* done;          /* cudaEvent_t, recorded after each launch */
    void* rows_host;     /* pinned: the boards in (int64 [largest, 70], or lean rows uint8 [largest, 508]) */
    void* rows;          /* device: the same */
    float* answers_host; /* pinned: the answers out ([largest, 1969], or lean [largest, 219]) */
    float* answers;      /* device: the same */
} FryLaneHandles;

int fry_lanes_create(const FryNetwork* network, const int* sizes, int sizes_count, int in_flight, int lean, int blocking_wait,
                     FryLanes** lanes);
int fry_lanes_destroy(FryLanes* lanes);
/* The first lane with no batch out (`GraphedBatches.free_lane`), or FRY_ERROR_STATE. */
int fry_lanes_free_lane(const FryLanes* lanes, int* lane);
int fry_lanes_handles(const FryLanes* lanes, int lane, FryLaneHandles* handles);
/* The graph executable (cudaGraphExec_t) of sizes[size_index] on a lane, for callers that replay it themselves. */
int fry_lanes_graph(const FryLanes* lanes, int lane, int size_index, void** graph_exec);
/* Copies `count` boards from the lane's pinned rows_host in, replays the smallest graph of at least `count` boards and
 * records the done event (`launch_filled`); *size is the graph's size. Returns at once. */
int fry_lanes_launch(FryLanes* lanes, int lane, int count, int* size);
/* Waits for the lane's batch (on the done event when blocking_wait, else on the stream) and copies its `count` answers
 * into answers_host (`collect`); *count is the batch's. */
int fry_lanes_collect(FryLanes* lanes, int lane, int* count);
/* Waits for every lane's batch and marks them collected without copying (`settle`). */
int fry_lanes_settle(FryLanes* lanes);

#ifdef __cplusplus
}
#endif

#endif /* FRY_B200_H */
