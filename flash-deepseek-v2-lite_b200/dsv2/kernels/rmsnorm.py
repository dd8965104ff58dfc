"""RMSNorm (reference: triton_kernels/rmsnorm.py:60-95)."""
from __future__ import annotations

import torch

from .. import ops


def rmsnorm_triton(hidden_states: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """y = x * rsqrt(mean(x^2) + eps) * w over the last dimension, fp32 math, output in
    x's dtype and shape.  Same checks and exception types as the reference
    (rmsnorm.py:62-76): bf16 or fp16 activations, a bf16, fp16 or fp32 weight; this build
    also needs a last dimension that is a multiple of 8 and at most 4096."""
    if hidden_states.device.type != "cuda":
        raise NotImplementedError("rmsnorm_triton requires CUDA tensor")
    if hidden_states.dtype not in (torch.bfloat16, torch.float16):
        raise NotImplementedError("rmsnorm_triton only supports bf16/fp16 input")
    if weight.dtype not in (torch.bfloat16, torch.float16, torch.float32):
        raise NotImplementedError("rmsnorm_triton only supports bf16/fp16/fp32 weight")
    if not weight.is_contiguous():
        raise NotImplementedError("rmsnorm_triton requires contiguous weight")
    x = hidden_states
    shape = x.shape
    n_cols = int(shape[-1])
    x_2d = x.view(-1, n_cols)
    if x_2d.stride(1) != 1:
        raise NotImplementedError("rmsnorm_triton requires last dimension to be contiguous")
    if n_cols % 8 or n_cols > 4096 or weight.numel() != n_cols:
        raise NotImplementedError(f"rmsnorm_triton: unsupported row length {n_cols}")
    y = torch.empty((x_2d.shape[0], n_cols), device=x.device, dtype=x.dtype)
    ops.rmsnorm(x_2d, weight, float(eps), y)
    return y.reshape(shape)
