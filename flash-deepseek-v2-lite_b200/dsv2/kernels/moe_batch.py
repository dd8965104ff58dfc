"""Batch-family routed MoE (reference: triton_kernels/moe_batch.py).

The reference buckets routes by expert with atomics and runs grouped Triton GEMMs
(moe_batch.py:390-557) after timing 15 tile candidates at warm-up (:596-657).  Here the
bucketing is stable (routes of an expert in token order), the GEMMs are the tcgen05/TMEM
grouped kernels of libdsv2 with a static tile choice, and there is no runtime autotune.
"""
from __future__ import annotations

import torch

from .. import ops
from ._moe import PackedRoutedExperts, pack_routed_experts, routed_moe

__all__ = ["PackedRoutedExperts", "pack_routed_experts", "packed_routed_moe", "batched_grouped_routed_moe"]


def batched_grouped_routed_moe(x: torch.Tensor, topk_ids: torch.Tensor, topk_weight: torch.Tensor,
                               packed: PackedRoutedExperts, output_dtype: torch.dtype | None = None) -> torch.Tensor:
    """Routed-expert MoE output [B, H] for x [B, H] bf16, topk_ids [B, 6] (int64 or int32),
    topk_weight [B, 6]; output_dtype bf16 (default: x's dtype) or fp32
    (moe_batch.py:402-422)."""
    return routed_moe("batched_grouped_routed_moe", x, topk_ids, topk_weight, packed, output_dtype,
                      ops.FAMILY_BATCH)


def packed_routed_moe(x: torch.Tensor, topk_ids: torch.Tensor, topk_weight: torch.Tensor,
                      packed: PackedRoutedExperts, output_dtype: torch.dtype | None = None) -> torch.Tensor:
    """Entry point of the batch MoE (moe_batch.py:390-399).  The reference drops to its
    eager loop for non-CUDA or non-2-D inputs; this build raises instead."""
    return batched_grouped_routed_moe(x, topk_ids, topk_weight, packed, output_dtype=output_dtype)
