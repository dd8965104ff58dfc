"""Small-family routed MoE, weight-streaming GEMV kernels (reference: triton_kernels/moe_small_gemv.py).

Semantics are those of the model's MoE (gate = W_gate x, up = W_up x, h = silu(gate) * up),
which is what the HF module computes.  The reference's small-batch Triton kernels read
the packed [gate; up] rows as consecutive blocks (moe_small_gemv.py:87-103, :235-251),
so their "up" operand is not the up projection; that behaviour is not reproduced.
"""
from __future__ import annotations

import torch

from .. import ops
from ._moe import PackedRoutedExperts, pack_routed_experts, routed_moe

__all__ = ["PackedRoutedExperts", "pack_routed_experts", "grouped_routed_moe",
           "batched_grouped_routed_moe_route_gemv"]


def grouped_routed_moe(x: torch.Tensor, topk_ids: torch.Tensor, topk_weight: torch.Tensor,
                       packed: PackedRoutedExperts, output_dtype: torch.dtype | None = None) -> torch.Tensor:
    """Single-token decode MoE: x [1, H], topk ids/weights [1, topk] -> [1, H]
    (moe_small_gemv.py:517-614)."""
    if x.ndim != 2 or x.shape[0] != 1:
        raise NotImplementedError("grouped_routed_moe only supports single-token decode")
    if topk_ids.ndim != 2 or topk_ids.shape[0] != 1:
        raise NotImplementedError("topk_ids must have shape [1, topk]")
    return routed_moe("grouped_routed_moe", x, topk_ids, topk_weight, packed, output_dtype, ops.FAMILY_SMALL)


def batched_grouped_routed_moe_route_gemv(x: torch.Tensor, topk_ids: torch.Tensor, topk_weight: torch.Tensor,
                                          packed: PackedRoutedExperts,
                                          output_dtype: torch.dtype | None = None) -> torch.Tensor:
    """Small-batch MoE: x [B, H], topk ids/weights [B, topk] -> [B, H]
    (moe_small_gemv.py:430-514).  Each expert's weights are streamed once per call for
    all of its routes (the reference re-reads them per route)."""
    return routed_moe("batched_grouped_routed_moe_route_gemv", x, topk_ids, topk_weight, packed,
                      output_dtype, ops.FAMILY_SMALL)
