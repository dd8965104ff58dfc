"""Small-family (weight-streaming GEMV) MLA decode attention
(reference: triton_kernels/attention_decode_small.py)."""
from __future__ import annotations

import torch

from .. import ops
from ._attention import AttentionDecodeWorkspace, AttentionPackedWeights, mla_decode_layer, pack_attention_weights

__all__ = ["AttentionPackedWeights", "AttentionDecodeWorkspace", "pack_attention_weights",
           "attention_decode_only_triton", "attention_decode_small_batch_triton"]


def attention_decode_only_triton(hidden_states: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                                 position_ids: torch.Tensor, cache_position: torch.Tensor,
                                 key_cache: torch.Tensor, value_cache: torch.Tensor | None,
                                 packed: AttentionPackedWeights, softmax_scale: float) -> torch.Tensor:
    """Single-token decode attention, hidden_states [1, 1, 2048] -> [1, 1, 2048]
    (attention_decode_small.py:553-674).  key_cache is the latent cache [1, S, 576];
    value_cache is ignored; cos/sin are [max_position, >= 32] rope tables (fp32 used
    as is, other dtypes converted per call)."""
    return mla_decode_layer("attention_decode_only_triton", hidden_states, cos, sin, position_ids,
                            cache_position, key_cache, value_cache, packed, softmax_scale, ops.FAMILY_SMALL,
                            single_row=True)


def attention_decode_small_batch_triton(hidden_states: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                                        position_ids: torch.Tensor, cache_position: torch.Tensor,
                                        key_cache: torch.Tensor, value_cache: torch.Tensor | None,
                                        packed: AttentionPackedWeights, softmax_scale: float) -> torch.Tensor:
    """Small-batch decode attention, hidden_states [B, 1, 2048] -> [B, 1, 2048]
    (attention_decode_small.py:932-1070).  cache_position may hold one position or one
    per row (ragged batch)."""
    return mla_decode_layer("attention_decode_small_batch_triton", hidden_states, cos, sin, position_ids,
                            cache_position, key_cache, value_cache, packed, softmax_scale, ops.FAMILY_SMALL,
                            single_row=False)
