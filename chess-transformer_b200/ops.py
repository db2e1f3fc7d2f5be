"""The reference's torch custom ops, one by one, on libfry_b200.so (torch.library ops in the `fry` namespace).

Each keeps the reference op's name, argument meaning, output shapes and dtypes (model/int8_blocks.py:132-251,
model/fused_blocks.py:104-177,308-318,397-411,495-512,743-779) and runs on the caller's current CUDA stream, so the ops
can be recorded in CUDA graphs and seen through by torch.compile (each has a fake implementation). CPU tensors are
refused with FryError: there is no CPU path.
"""
import ctypes

import torch

from .library import FryError, FryHeads, library

HADAMARD_BLOCK = 32


def _stream(tensor: torch.Tensor) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(tensor.device).cuda_stream)


def _ptr(tensor: torch.Tensor | None) -> ctypes.c_void_p | None:
    return None if tensor is None else ctypes.c_void_p(tensor.data_ptr())


def _cuda(name: str, *tensors: torch.Tensor | None) -> None:
    for tensor in tensors:
        if tensor is not None and not tensor.is_cuda:
            raise FryError(f"{name} runs on the GPU only; got a tensor on {tensor.device}")


def _dtype(name: str, tensor: torch.Tensor | None, dtype: torch.dtype, what: str) -> None:
    if tensor is not None and tensor.dtype != dtype:
        raise FryError(f"{name}: {what} must be {dtype}, got {tensor.dtype}")


@torch.library.custom_op("fry::int8_linear", mutates_args=())
def int8_linear(x: torch.Tensor, x_scale: torch.Tensor, weight: torch.Tensor, weight_scale: torch.Tensor, bias: torch.Tensor | None,
                residual: torch.Tensor | None, gated: bool, matmul: str, original: torch.Tensor | None = None,
                residual_scale: torch.Tensor | None = None, input_scale: torch.Tensor | None = None) -> torch.Tensor:
    """`chess::int8_linear` (model/int8_blocks.py:132-139). `matmul` names the reference's tile table; one kernel serves all."""
    _cuda("int8_linear", x, x_scale, weight, weight_scale, bias, residual, original)
    _dtype("int8_linear", x, torch.int8, "x")
    _dtype("int8_linear", weight, torch.int8, "weight")
    rows, K = weight.shape
    N = rows // 2 if gated else rows
    x = x.contiguous()
    M = x.numel() // K
    out = torch.empty(*x.shape[:-1], N, device=x.device, dtype=torch.float16)
    residual = residual.contiguous() if residual is not None else None
    original = original.contiguous() if original is not None else None
    x_scale, weight, weight_scale = x_scale.contiguous().float(), weight.contiguous(), weight_scale.contiguous().float()
    bias = bias.half().contiguous() if bias is not None else None
    library().fry_int8_linear(_ptr(x), _ptr(x_scale), _ptr(weight), _ptr(weight_scale), _ptr(bias), _ptr(residual), _ptr(original),
                              _ptr(residual_scale), _ptr(input_scale), _ptr(out), M, N, K, int(gated), _stream(x))
    return out


@int8_linear.register_fake
def _(x, x_scale, weight, weight_scale, bias, residual, gated, matmul, original=None, residual_scale=None, input_scale=None):
    return x.new_empty(*x.shape[:-1], weight.shape[0] // 2 if gated else weight.shape[0], dtype=torch.float16)


@torch.library.custom_op("fry::int8_linear_normed", mutates_args=())
def int8_linear_normed(x: torch.Tensor, gain: torch.Tensor, eps: float, weight: torch.Tensor, weight_scale: torch.Tensor,
                       bias: torch.Tensor | None, gated: bool) -> torch.Tensor:
    """`chess::norm_quant` then `chess::int8_linear` (model/int8_blocks.py:191-193, :132-139) as one kernel, the pair
    `Int8Block.forward` runs for ln1 -> projection and ln2 -> gate_up (model/int8_blocks.py:274-288); the same bits as
    `int8_linear(*norm_quant(x, gain, eps), ...)`. x fp16 [..., 768]."""
    _cuda("int8_linear_normed", x, gain, weight, weight_scale, bias)
    _dtype("int8_linear_normed", x, torch.float16, "x")
    _dtype("int8_linear_normed", weight, torch.int8, "weight")
    rows, K = weight.shape
    N = rows // 2 if gated else rows
    x = x.contiguous()
    M = x.numel() // K
    out = torch.empty(*x.shape[:-1], N, device=x.device, dtype=torch.float16)
    bias = bias.half().contiguous() if bias is not None else None
    library().fry_int8_linear_normed(_ptr(x), _ptr(gain.half().contiguous()), eps, _ptr(weight.contiguous()),
                                     _ptr(weight_scale.contiguous().float()), _ptr(bias), _ptr(out), M, N, K, int(gated), _stream(x))
    return out


@int8_linear_normed.register_fake
def _(x, gain, eps, weight, weight_scale, bias, gated):
    return x.new_empty(*x.shape[:-1], weight.shape[0] // 2 if gated else weight.shape[0], dtype=torch.float16)


@torch.library.custom_op("fry::int8_matmul_i32", mutates_args=())
def int8_matmul_i32(x: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """The int32 sums x . weight^T of the int8 tensor-core kernel (what int8_linear's epilogue starts from)."""
    _cuda("int8_matmul_i32", x, weight)
    x, weight = x.contiguous(), weight.contiguous()
    N, K = weight.shape
    M = x.numel() // K
    out = torch.empty(*x.shape[:-1], N, device=x.device, dtype=torch.int32)
    library().fry_int8_matmul_i32(_ptr(x), _ptr(weight), _ptr(out), M, N, K, _stream(x))
    return out


@int8_matmul_i32.register_fake
def _(x, weight):
    return x.new_empty(*x.shape[:-1], weight.shape[0], dtype=torch.int32)


@torch.library.custom_op("fry::int8_matmul_scaled_bf16", mutates_args=())
def int8_matmul_scaled_bf16(x: torch.Tensor, x_scale: torch.Tensor, weight: torch.Tensor, weight_scale: torch.Tensor) -> torch.Tensor:
    """The benchmark's isolated int8 GEMM: bf16((acc * x_scale[m]) * weight_scale[n]), acc = x . weight^T in int32, on the
    int8 tensor-core kernel. x int8 [..., K], weight int8 [N, K], scales fp32."""
    _cuda("int8_matmul_scaled_bf16", x, x_scale, weight, weight_scale)
    _dtype("int8_matmul_scaled_bf16", x, torch.int8, "x")
    _dtype("int8_matmul_scaled_bf16", weight, torch.int8, "weight")
    x, weight = x.contiguous(), weight.contiguous()
    N, K = weight.shape
    M = x.numel() // K
    out = torch.empty(*x.shape[:-1], N, device=x.device, dtype=torch.bfloat16)
    library().fry_int8_matmul_scaled_bf16(_ptr(x), _ptr(x_scale.contiguous().float()), _ptr(weight), _ptr(weight_scale.contiguous().float()),
                                          _ptr(out), M, N, K, _stream(x))
    return out


@int8_matmul_scaled_bf16.register_fake
def _(x, x_scale, weight, weight_scale):
    return x.new_empty(*x.shape[:-1], weight.shape[0], dtype=torch.bfloat16)


@torch.library.custom_op("fry::attention_bf16", mutates_args=())
def attention_bf16(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, heads: int) -> torch.Tensor:
    """The benchmark's isolated attention: softmax(q k^T / 8) v per sequence and head, q, k, v bf16 [B, 64, heads * 64]."""
    _cuda("attention_bf16", q, k, v)
    for name, tensor in (("q", q), ("k", k), ("v", v)):
        _dtype("attention_bf16", tensor, torch.bfloat16, name)
    if q.dim() != 3 or q.shape != k.shape or q.shape != v.shape or q.shape[-1] % heads != 0:
        raise FryError(f"attention_bf16 takes q, k and v of one shape [B, seq, heads * head_dim], got {tuple(q.shape)}")
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    B, seq, width = q.shape
    out = torch.empty_like(q)
    library().fry_attention_bf16(_ptr(q), _ptr(k), _ptr(v), _ptr(out), B, heads, seq, width // heads, _stream(q))
    return out


@attention_bf16.register_fake
def _(q, k, v, heads):
    return torch.empty_like(q)


@torch.library.custom_op("fry::norm_quant", mutates_args=())
def norm_quant(x: torch.Tensor, gain: torch.Tensor, eps: float) -> tuple[torch.Tensor, torch.Tensor]:
    """`chess::norm_quant` (model/int8_blocks.py:191-193): int8 rows of RMSNorm(x) * gain and their scales."""
    _cuda("norm_quant", x, gain)
    _dtype("norm_quant", x, torch.float16, "x")
    x = x.contiguous()
    D = x.shape[-1]
    q = torch.empty(x.shape, device=x.device, dtype=torch.int8)
    scale = torch.empty(x.shape[:-1], device=x.device, dtype=torch.float32)
    library().fry_norm_quant(_ptr(x), _ptr(gain.contiguous()), eps, _ptr(q), _ptr(scale), x.numel() // D, D, _stream(x))
    return q, scale


@norm_quant.register_fake
def _(x, gain, eps):
    return x.new_empty(x.shape, dtype=torch.int8), x.new_empty(x.shape[:-1], dtype=torch.float32)


@torch.library.custom_op("fry::mix_norm_quant", mutates_args=())
def mix_norm_quant(x: torch.Tensor, original: torch.Tensor, residual_scale: torch.Tensor, input_scale: torch.Tensor, gain: torch.Tensor,
                   eps: float) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """`chess::mix_norm_quant` (model/int8_blocks.py:201-207): the block input mixed with the embedding, then norm_quant."""
    _cuda("mix_norm_quant", x, original, residual_scale, input_scale, gain)
    x, original = x.contiguous(), original.contiguous()
    D = x.shape[-1]
    mixed = torch.empty_like(x, dtype=torch.float16)
    q = torch.empty(x.shape, device=x.device, dtype=torch.int8)
    scale = torch.empty(x.shape[:-1], device=x.device, dtype=torch.float32)
    library().fry_mix_norm_quant(_ptr(x), _ptr(original), _ptr(residual_scale), _ptr(input_scale), _ptr(gain.contiguous()), eps,
                                 _ptr(mixed), _ptr(q), _ptr(scale), x.numel() // D, D, _stream(x))
    return mixed, q, scale


@mix_norm_quant.register_fake
def _(x, original, residual_scale, input_scale, gain, eps):
    return x.new_empty(x.shape, dtype=torch.float16), x.new_empty(x.shape, dtype=torch.int8), x.new_empty(x.shape[:-1], dtype=torch.float32)


@torch.library.custom_op("fry::rotate_quant", mutates_args=())
def rotate_quant(h: torch.Tensor, hadamard_signs: torch.Tensor, width: int) -> tuple[torch.Tensor, torch.Tensor]:
    """`chess::rotate_quant` (model/int8_blocks.py:234-246). The kernel applies Sylvester's 32x32 signs itself, the matrix
    the reference passes as hadamard_signs (`hadamard(32)`, model/int8_blocks.py:54-58); any other matrix is refused."""
    _cuda("rotate_quant", h)
    if tuple(hadamard_signs.shape) != (HADAMARD_BLOCK, HADAMARD_BLOCK):
        raise FryError(f"rotate_quant rotates by 32x32 Hadamard blocks, got signs of shape {tuple(hadamard_signs.shape)}")
    h = h.contiguous()
    hidden = h.shape[-1]
    q = torch.empty(*h.shape[:-1], width, device=h.device, dtype=torch.int8)
    scale = torch.empty(h.shape[:-1], device=h.device, dtype=torch.float32)
    library().fry_rotate_quant(_ptr(h), _ptr(q), _ptr(scale), h.numel() // hidden, hidden, width, _stream(h))
    return q, scale


@rotate_quant.register_fake
def _(h, hadamard_signs, width):
    return h.new_empty(*h.shape[:-1], width, dtype=torch.int8), h.new_empty(h.shape[:-1], dtype=torch.float32)


@torch.library.custom_op("fry::template_attention", mutates_args=())
def template_attention(projected: torch.Tensor, templates: torch.Tensor, q_gain: torch.Tensor, k_gain: torch.Tensor, heads: int,
                       kv_heads: int, dq: int, dv: int, templates_count: int, eps: float) -> torch.Tensor:
    """`chess::template_attention` (model/fused_blocks.py:104-171): projected [B, 70, q|k|v|mix] -> [B, 70, heads * dv]."""
    _cuda("template_attention", projected, templates, q_gain, k_gain)
    projected = projected.contiguous()
    B, T, _ = projected.shape
    if T != 70:
        raise FryError(f"template_attention takes 70 tokens a position, got {T}")
    out = projected.new_empty(B, T, heads * dv)
    paired = pair_templates(templates)
    library().fry_template_attention(_ptr(projected), _ptr(paired), _ptr(q_gain.contiguous()), _ptr(k_gain.contiguous()),
                                     _ptr(out), B, heads, kv_heads, dq, dv, templates_count, eps, _stream(projected))
    return out


def pair_templates(templates: torch.Tensor) -> torch.Tensor:
    """The templates [8, 64, 64] re-laid as [64, 64, 8] for the attention kernel (the reference's `paired_templates`,
    model/attention_cuda.py:412-434). Paired afresh on every call here, on the current stream, so that the op records
    into CUDA graphs; the network pairs its templates once."""
    _cuda("pair_templates", templates)
    if tuple(templates.shape) != (8, 64, 64) or templates.dtype != torch.float16:
        raise FryError(f"the attention takes 8 fp16 templates of 64 x 64, got {tuple(templates.shape)} {templates.dtype}")
    templates = templates.contiguous()
    paired = templates.new_empty(64, 64, 8)
    library().fry_pair_templates(_ptr(templates), _ptr(paired), 8, _stream(templates))
    return paired


@template_attention.register_fake
def _(projected, templates, q_gain, k_gain, heads, kv_heads, dq, dv, templates_count, eps):
    B, T, _ = projected.shape
    return projected.new_empty(B, T, heads * dv)


@torch.library.custom_op("fry::linear", mutates_args=())
def linear(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None, residual: torch.Tensor | None = None,
           gated: bool = False, accumulate_fp32: bool = False, original: torch.Tensor | None = None,
           residual_scale: torch.Tensor | None = None, input_scale: torch.Tensor | None = None) -> torch.Tensor:
    """`chess::linear` (model/fused_blocks.py:308-313) for fp16 x and weight [K, N] as the reference stores it ([K, 2N],
    gate columns then up columns, gated): fp32 accumulation (the reference accumulates fp16 inputs in fp16 unless
    accumulate_fp32), fp16 out, or fp32 out with accumulate_fp32; the gated and input-mixing forms (the fp16 blocks')
    in fp16."""
    _cuda("linear", x, weight, bias, residual, original, residual_scale, input_scale)
    _dtype("linear", x, torch.float16, "x")
    if gated or original is not None:  # the fp16 blocks' forms (fp16 out)
        if accumulate_fp32:
            raise FryError("fry::linear gives its gated and input-mixing forms in fp16 only")
        K, width = weight.shape
        N = width // 2 if gated else width
        x = x.contiguous()
        M = x.numel() // K
        out = x.new_empty(*x.shape[:-1], N, dtype=torch.float16)
        bias = bias.half().contiguous() if bias is not None else None
        residual = residual.contiguous() if residual is not None else None
        original = original.contiguous() if original is not None else None
        library().fry_linear_full(_ptr(x), _ptr(weight.t().contiguous()), _ptr(bias), _ptr(residual), _ptr(original), _ptr(residual_scale),
                                  _ptr(input_scale), _ptr(out), M, N, K, int(gated), _stream(x))
        return out
    K, N = weight.shape
    x = x.contiguous()
    M = x.numel() // K
    out = x.new_empty(*x.shape[:-1], N, dtype=torch.float32 if accumulate_fp32 else torch.float16)
    if bias is not None:
        bias = bias.float().contiguous() if accumulate_fp32 else bias.half().contiguous()
    weight_nk = weight.t().contiguous()
    residual = residual.contiguous() if residual is not None else None
    library().fry_linear(_ptr(x), _ptr(weight_nk), _ptr(bias), _ptr(residual), _ptr(out), M, N, K, int(accumulate_fp32), _stream(x))
    return out


@linear.register_fake
def _(x, weight, bias=None, residual=None, gated=False, accumulate_fp32=False, original=None, residual_scale=None, input_scale=None):
    return x.new_empty(*x.shape[:-1], weight.shape[1] // 2 if gated else weight.shape[1], dtype=torch.float32 if accumulate_fp32 else x.dtype)


@torch.library.custom_op("fry::linear_norm_quant", mutates_args=())
def linear_norm_quant(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None, residual: torch.Tensor | None, gain: torch.Tensor,
                      eps: float) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """`chess::linear` (fp16, weight [K, N] as the reference stores it) then `chess::norm_quant` of its output
    (model/int8_blocks.py:191-193, 274-288) as one kernel: (out, q, scale). out equals `linear`'s bit for bit; q and scale
    equal `norm_quant(out, gain, eps)` to within its rounding. N a multiple of 256 up to 1024."""
    _cuda("linear_norm_quant", x, weight, bias, residual, gain)
    _dtype("linear_norm_quant", x, torch.float16, "x")
    K, N = weight.shape
    x = x.contiguous()
    M = x.numel() // K
    out = x.new_empty(*x.shape[:-1], N, dtype=torch.float16)
    q = x.new_empty(*x.shape[:-1], N, dtype=torch.int8)
    scale = x.new_empty(x.shape[:-1], dtype=torch.float32)
    bias = bias.half().contiguous() if bias is not None else None
    residual = residual.contiguous() if residual is not None else None
    library().fry_linear_norm_quant(_ptr(x), _ptr(weight.t().contiguous()), _ptr(bias), _ptr(residual), _ptr(out), _ptr(gain.half().contiguous()),
                                    eps, _ptr(q), _ptr(scale), M, N, K, _stream(x))
    return out, q, scale


@linear_norm_quant.register_fake
def _(x, weight, bias, residual, gain, eps):
    shape = (*x.shape[:-1], weight.shape[1])
    return x.new_empty(shape, dtype=torch.float16), x.new_empty(shape, dtype=torch.int8), x.new_empty(x.shape[:-1], dtype=torch.float32)


@torch.library.custom_op("fry::board_embedding", mutates_args=())
def board_embedding(boards: torch.Tensor, embed: torch.Tensor, position: torch.Tensor, table: torch.Tensor) -> torch.Tensor:
    """`chess::board_embedding` (model/fused_blocks.py:495-507): boards [B, 70] -> [B, 70, D] fp16, the 23 square-feature
    rows of `SquareFeatures.indices` found in the kernel (the reference's rays and jumps tables are built in)."""
    _cuda("board_embedding", boards, embed, position, table)
    boards = boards.long().contiguous()
    B, T = boards.shape
    D = table.shape[1]
    out = table.new_empty(B, T, D)
    library().fry_board_embedding(_ptr(boards), _ptr(embed.contiguous()), _ptr(position.contiguous()), _ptr(table.contiguous()), _ptr(out),
                                  B, D, _stream(boards))
    return out


@board_embedding.register_fake
def _(boards, embed, position, table):
    return table.new_empty(*boards.shape, table.shape[1])


def heads_struct(ln_gain, a_weight, a_bias, narrow_weight, narrow_bias, hidden_weight, hidden_bias, out_weight, out_bias) -> FryHeads:
    return FryHeads(_ptr(ln_gain), _ptr(a_weight), _ptr(a_bias), _ptr(narrow_weight), _ptr(narrow_bias), _ptr(hidden_weight),
                    _ptr(hidden_bias), _ptr(out_weight), _ptr(out_bias), out_weight.shape[0])


@torch.library.custom_op("fry::heads", mutates_args=())
def heads(stream: torch.Tensor, ln_gain: torch.Tensor, a_weight: torch.Tensor, a_bias: torch.Tensor, narrow_weight: torch.Tensor,
          narrow_bias: torch.Tensor, hidden_weight: torch.Tensor, hidden_bias: torch.Tensor, out_weight: torch.Tensor,
          out_bias: torch.Tensor, eps: float) -> torch.Tensor:
    """The heads from the last block's stream to the answer rows [B, 1969] (the reference's `heads` op,
    model/fused_blocks.py:743-774, computes the same rows from its own folded weights). a_weight is [N, K] fp16:
    (W_f^T W_t / sqrt d)^T; narrow_weight [21, d] fp32; the eval head's layers as nn.Linear holds them, in fp32."""
    _cuda("heads", stream, ln_gain, a_weight, a_bias, narrow_weight, narrow_bias, hidden_weight, hidden_bias, out_weight, out_bias)
    stream = stream.contiguous()
    B, T, D = stream.shape
    rows = torch.empty(B, 1969, device=stream.device, dtype=torch.float32)
    lib = library()
    workspace = torch.empty(lib.fry_heads_workspace_bytes(B, D), device=stream.device, dtype=torch.uint8)
    weights = heads_struct(ln_gain, a_weight, a_bias, narrow_weight, narrow_bias, hidden_weight, hidden_bias, out_weight, out_bias)
    lib.fry_heads(_ptr(stream), ctypes.byref(weights), eps, _ptr(rows), _ptr(workspace), workspace.numel(), B, D, _stream(stream))
    return rows


@heads.register_fake
def _(stream, ln_gain, a_weight, a_bias, narrow_weight, narrow_bias, hidden_weight, hidden_bias, out_weight, out_bias, eps):
    return stream.new_empty(stream.shape[0], 1969, dtype=torch.float32)
