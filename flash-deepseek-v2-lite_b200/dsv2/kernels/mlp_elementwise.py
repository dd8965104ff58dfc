"""SiLU-and-multiply between the dense MLP GEMMs (reference: triton_kernels/mlp_elementwise.py:24-45)."""
from __future__ import annotations

import torch

from .. import ops


def silu_mul_triton(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """out = bf16(silu(gate) * up), fp32 math; a new tensor shaped like gate."""
    if gate.device.type != "cuda" or up.device.type != "cuda":
        raise NotImplementedError("silu_mul_triton requires CUDA tensors")
    if gate.shape != up.shape:
        raise ValueError("gate and up must have the same shape")
    if gate.dtype != torch.bfloat16 or up.dtype != torch.bfloat16:
        raise NotImplementedError("silu_mul_triton supports bf16 only")
    if not gate.is_contiguous() or not up.is_contiguous():
        raise NotImplementedError("silu_mul_triton requires contiguous inputs")
    if gate.numel() % 8:
        raise NotImplementedError("silu_mul_triton: element count must be a multiple of 8")
    out = torch.empty_like(gate)
    ops.silu_mul(gate, up, out)
    return out
