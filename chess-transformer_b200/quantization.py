"""GPTQ on the device: the drop-in for the reference's `gptq` (engine/quantization.py:76-99), which
`compute_int8_weights` (:104-140) calls for every int8 matmul of every block. One C-ABI call (fry_gptq) runs it in fp64
on the weight's GPU; the answer is the reference's (int8 [N, K], fp32 scale [N]) on that device.
"""
import ctypes

import torch

from .library import FryError, library

NOT_POSITIVE_DEFINITE = 6  # the device status code fry_gptq records


def gptq(weight: torch.Tensor, hessian: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """engine/quantization.py:76-99: (int8 weight, fp32 scale a row) of an N x K weight, each column's error spread over
    the later ones through the Hessian [K, K]. Both are taken as fp64 (as the reference takes them) on the weight's CUDA
    device. Raises FryError if the dampened Hessian is not positive definite, where the reference's
    torch.linalg.cholesky raises."""
    if weight.dim() != 2 or hessian.shape != (weight.shape[1], weight.shape[1]):
        raise ValueError(f"gptq takes weight [N, K] and hessian [K, K], got {tuple(weight.shape)} and {tuple(hessian.shape)}")
    device = weight.device if weight.is_cuda else torch.device("cuda")
    weight64 = weight.detach().to(device=device, dtype=torch.float64).contiguous()
    hessian64 = hessian.detach().to(device=device, dtype=torch.float64).contiguous()
    N, K = weight64.shape
    lib = library()
    integers = torch.empty(N, K, dtype=torch.int8, device=device)
    scale = torch.empty(N, dtype=torch.float32, device=device)
    workspace = torch.empty(lib.fry_gptq_workspace_bytes(N, K), dtype=torch.uint8, device=device)
    with torch.cuda.device(device):
        before = lib.device_status()
        stream = torch.cuda.current_stream(device)
        lib.fry_gptq(ctypes.c_void_p(weight64.data_ptr()), ctypes.c_void_p(hessian64.data_ptr()), N, K,
                     ctypes.c_void_p(integers.data_ptr()), ctypes.c_void_p(scale.data_ptr()), ctypes.c_void_p(workspace.data_ptr()),
                     workspace.numel(), ctypes.c_void_p(stream.cuda_stream))
        stream.synchronize()
        code, where = lib.device_status()
        if code == NOT_POSITIVE_DEFINITE and before[0] != NOT_POSITIVE_DEFINITE:
            lib.device_status(clear=True)
            raise FryError(f"gptq: the dampened Hessian is not positive definite (Cholesky pivot {where})")
    return integers, scale
