"""Batch-family (tcgen05/TMEM linears) MLA decode attention
(reference: triton_kernels/attention_decode_batch.py)."""
from __future__ import annotations

import torch

from .. import ops
from ._attention import AttentionDecodeWorkspace, AttentionPackedWeights, mla_decode_layer, pack_attention_weights

__all__ = ["AttentionPackedWeights", "AttentionDecodeWorkspace", "pack_attention_weights",
           "attention_decode_triton"]


def attention_decode_triton(hidden_states: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                            position_ids: torch.Tensor, cache_position: torch.Tensor,
                            key_cache: torch.Tensor, value_cache: torch.Tensor | None,
                            packed: AttentionPackedWeights, softmax_scale: float) -> torch.Tensor:
    """Batched decode attention, hidden_states [B, 1, 2048] -> [B, 1, 2048]
    (attention_decode_batch.py:672-846).  key_cache is the latent cache [B, S, 576];
    value_cache is ignored; cache_position holds one position or one per row."""
    return mla_decode_layer("attention_decode_triton", hidden_states, cos, sin, position_ids, cache_position,
                            key_cache, value_cache, packed, softmax_scale, ops.FAMILY_BATCH, single_row=False)
