"""The checkpoint's own network in fp64 on the GPU, for offline calibration of its int8 weights.

The reference rounds a checkpoint's weights by GPTQ over the input Hessians of each int8 matmul, summed while the fp32
checkpoint runs in fp64 on the calibration positions (`int8_weights`, engine/quantization.py:199-203: `load_model(...)
.half_except_heads(torch.float64)`, then `compute_int8_weights`, :122-140, whose hooks read the inputs of each block's
Q, mlp.gate_projection and mlp.down_projection, :103-119). `CalibrationNetwork` is that network: the blocks of
`TransformerBlock.forward` (model/model.py:71-99) after the input embedding (model/model.py:245-249), every weight
fp64, with the same module names, so `quantization.input_hessians` hooks it as the reference hooks its model. Only the
blocks run: the heads read nothing a Hessian needs. The square features' table rows come from the library's own kernel
(fry_square_feature_rows, the rows the forward's embedding sums).
"""
import ctypes
import math

import torch
import torch.nn.functional as F
from torch import nn

from .encoding import NUM_SQUARES, TOKENS_PER_BOARD
from .library import FryError, library

EPS = 1e-5  # every RMSNorm of the model (model/model.py:55-60)


def _linear(state: dict, name: str, device, bias: bool) -> nn.Linear:
    weight = state[name + ".weight"]
    layer = nn.Linear(weight.shape[1], weight.shape[0], bias=bias, device=device, dtype=torch.float64)
    with torch.no_grad():
        layer.weight.copy_(weight.to(device=device, dtype=torch.float64))
        if bias:
            layer.bias.copy_(state[name + ".bias"].to(device=device, dtype=torch.float64))
    return layer


class _SwiGLU(nn.Module):
    def __init__(self, state: dict, prefix: str, device):
        super().__init__()
        self.gate_projection = _linear(state, prefix + "gate_projection", device, bias=False)
        self.up_projection = _linear(state, prefix + "up_projection", device, bias=False)
        self.down_projection = _linear(state, prefix + "down_projection", device, bias=False)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.down_projection(F.silu(self.gate_projection(x)) * self.up_projection(x))


class CalibrationBlock(nn.Module):
    """One block in fp64: the input skip, ln1, Q/K/V with their RMSNorms, template-biased grouped-query attention,
    combine_heads, ln2 and the SwiGLU MLP (model/model.py:71-99)."""

    def __init__(self, state: dict, layer: int, heads: int, kv_heads: int, dq: int, dv: int, templates_count: int, device):
        super().__init__()
        p = f"encoder.{layer}."
        vector = lambda name: state[p + name].to(device=device, dtype=torch.float64)
        self.heads, self.kv_heads, self.dq, self.dv, self.templates_count = heads, kv_heads, dq, dv, templates_count
        self.Q, self.K, self.V = (_linear(state, p + name, device, bias=True) for name in ("Q", "K", "V"))
        self.template_mix = _linear(state, p + "template_mix", device, bias=True)
        self.combine_heads = _linear(state, p + "combine_heads", device, bias=True)
        self.mlp = _SwiGLU(state, p + "mlp.", device)
        self.q_gain, self.k_gain = vector("q_norm.weight"), vector("k_norm.weight")
        self.ln1_gain, self.ln2_gain = vector("ln1.weight"), vector("ln2.weight")
        self.residual_scale, self.input_scale = vector("residual_scale"), vector("input_scale")

    def forward(self, x: torch.Tensor, templates: torch.Tensor, original: torch.Tensor) -> torch.Tensor:
        B, T, d = x.shape
        residual = self.residual_scale * x + self.input_scale * original
        normed = F.rms_norm(residual, (d,), self.ln1_gain, EPS)
        q = F.rms_norm(self.Q(normed).reshape(B, T, self.heads, self.dq), (self.dq,), self.q_gain, EPS).transpose(1, 2)
        k = F.rms_norm(self.K(normed).reshape(B, T, self.kv_heads, self.dq), (self.dq,), self.k_gain, EPS).transpose(1, 2)
        v = self.V(normed).reshape(B, T, self.kv_heads, self.dv).transpose(1, 2)
        group = self.heads // self.kv_heads
        k, v = k.repeat_interleave(group, dim=1), v.repeat_interleave(group, dim=1)
        scores = q @ k.transpose(-2, -1) / math.sqrt(self.dq)
        mix = self.template_mix(normed[:, :NUM_SQUARES]).reshape(B, NUM_SQUARES, self.heads, self.templates_count)
        bias = torch.einsum("biht,tij->bhij", mix, templates)
        scores = scores + F.pad(bias, (0, T - NUM_SQUARES, 0, T - NUM_SQUARES))
        attended = (torch.softmax(scores, dim=-1) @ v).transpose(1, 2).reshape(B, T, d)
        residual = residual + self.combine_heads(attended)
        return residual + self.mlp(F.rms_norm(residual, (d,), self.ln2_gain, EPS))


class CalibrationNetwork(nn.Module):
    """The checkpoint's blocks in fp64 on `device` (a CUDA device). forward(boards int64 [B, 70]) -> the last block's
    output [B, 70, d] fp64."""

    def __init__(self, state: dict, geometry: dict, device: torch.device | str | None = None):
        super().__init__()
        device = torch.device(device if device is not None else "cuda")
        if device.type != "cuda":
            raise FryError("the calibration network runs on a CUDA device only")
        self.device = device
        wide = lambda name: state[name].to(device=device, dtype=torch.float64)
        self.embed, self.position, self.table, self.templates = wide("embed.weight"), wide("position_embed"), wide("square_features.table"), wide("templates")
        g = geometry
        self.encoder = nn.ModuleList([CalibrationBlock(state, i, g["heads"], g["kv_heads"], dq, g["dv"], g["templates"], device)
                                      for i, dq in enumerate(g["dqs"])])

    def embedding(self, boards: torch.Tensor) -> torch.Tensor:
        """embed[token] + position + the square features' 23 table rows summed, padded over the metadata tokens
        (model/model.py:171-174,245-249), in fp64."""
        boards = boards.to(device=self.device, dtype=torch.int64).contiguous()
        B = boards.shape[0]
        rows = torch.empty(B, NUM_SQUARES, 23, dtype=torch.int32, device=self.device)
        library().fry_square_feature_rows(ctypes.c_void_p(boards.data_ptr()), B, ctypes.c_void_p(rows.data_ptr()),
                                          ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream))
        features = self.table[rows.long()].sum(dim=-2)
        return self.embed[boards] + self.position + F.pad(features, (0, 0, 0, TOKENS_PER_BOARD - NUM_SQUARES))

    @torch.no_grad()
    def forward(self, boards: torch.Tensor) -> torch.Tensor:
        original = self.embedding(boards)
        x = original
        for block in self.encoder:
            x = block(x, self.templates, original)
        return x
