"""Decode-step glue around attention (reference: triton_kernels/attention_prepost.py)."""
from __future__ import annotations

import torch

from .. import ops


def copy_single_token_to_cache(src: torch.Tensor, dst: torch.Tensor, cache_position: torch.Tensor) -> None:
    """dst[b, h, pos, :] = src[b, h, 0, :] in place (attention_prepost.py:113-149).
    cache_position holds one position (the reference's case) or one per row; a position
    outside [0, S) sets the device error word and skips that row."""
    if src.device.type != "cuda" or dst.device.type != "cuda":
        raise NotImplementedError("copy_single_token_to_cache requires CUDA tensors")
    if src.ndim != 4 or dst.ndim != 4 or src.shape[2] != 1 or src.shape[0] != dst.shape[0]:
        raise NotImplementedError("copy_single_token_to_cache only supports [B, H, 1, D] -> [B, H, S, D]")
    if src.shape[1] != dst.shape[1] or src.shape[3] != dst.shape[3]:
        raise NotImplementedError("copy_single_token_to_cache: head count and head dim must match")
    if src.dtype != dst.dtype:
        raise ValueError("src and dst dtype must match")
    if src.element_size() not in (2, 4):
        raise NotImplementedError("copy_single_token_to_cache supports 2- and 4-byte elements")
    if cache_position.device.type != "cuda" or cache_position.numel() not in (1, src.shape[0]):
        raise ValueError("cache_position must be a CUDA tensor with one element (or one per row)")
    if cache_position.dtype != torch.long:
        raise ValueError("cache_position must be int64")
    ops.copy_token_to_cache(src, dst, cache_position.reshape(-1))


def prepare_decode_inputs_triton(cache_position: torch.Tensor, attention_mask: torch.Tensor,
                                 position_ids: torch.Tensor, attention_mask_index: torch.Tensor) -> None:
    """attention_mask[b, s] = (attention_mask_index[s] <= pos); position_ids[b, 0] = pos,
    in place (attention_prepost.py:152-188)."""
    if cache_position.device.type != "cuda":
        raise NotImplementedError("prepare_decode_inputs_triton requires CUDA tensors")
    if cache_position.numel() != 1:
        raise ValueError("cache_position must have one element")
    if attention_mask.ndim != 2:
        raise ValueError("attention_mask must have shape [batch, max_cache_len]")
    if position_ids.ndim != 2 or position_ids.shape[0] != attention_mask.shape[0] or position_ids.shape[1] != 1:
        raise ValueError("position_ids must have shape [batch, 1]")
    if attention_mask_index.ndim != 1 or attention_mask_index.shape[0] != attention_mask.shape[1]:
        raise ValueError("attention_mask_index must be 1D with length max_cache_len")
    if (attention_mask.dtype != torch.long or position_ids.dtype != torch.long
            or attention_mask_index.dtype != torch.long or cache_position.dtype != torch.long):
        raise ValueError("prepare_decode_inputs_triton requires int64 tensors")
    if attention_mask.stride(1) != 1 or not attention_mask_index.is_contiguous():
        raise NotImplementedError("prepare_decode_inputs_triton requires contiguous mask rows")
    ops.prepare_decode_inputs(cache_position, attention_mask, position_ids, attention_mask_index,
                              int(attention_mask.shape[0]), int(attention_mask.shape[1]))


def residual_add_triton(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """a + b with fp32 math, rounded to the inputs' dtype (bf16 or fp16), into a new tensor
    (attention_prepost.py:191-223)."""
    if a.device.type != "cuda" or b.device.type != "cuda":
        raise NotImplementedError("residual_add_triton requires CUDA tensors")
    if a.shape != b.shape:
        raise ValueError("a and b must have the same shape")
    if a.dtype not in (torch.bfloat16, torch.float16) or b.dtype != a.dtype:
        raise NotImplementedError("residual_add_triton supports bf16/fp16 with same dtype")
    if not a.is_contiguous() or not b.is_contiguous():
        raise NotImplementedError("residual_add_triton requires contiguous inputs")
    if a.numel() % 8:
        raise NotImplementedError("residual_add_triton: element count must be a multiple of 8")
    out = torch.empty_like(a)
    ops.residual_add(a, b, out)
    return out
