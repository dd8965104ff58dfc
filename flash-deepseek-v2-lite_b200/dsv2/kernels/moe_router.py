"""Router softmax + top-6 (reference: triton_kernels/moe_router.py:63-86)."""
from __future__ import annotations

import torch

from .. import ops


def router_softmax_topk6_triton(logits: torch.Tensor, scaling: float) -> tuple[torch.Tensor, torch.Tensor]:
    """softmax over the expert logits, the 6 largest probabilities in descending order
    (lowest index first on ties), weights = prob * scaling.  Returns (int64 ids [R, 6],
    fp32 weights [R, 6]).  The reference is specialised to [1, 64]; this build takes any
    number of rows R of 6..64 experts."""
    if logits.device.type != "cuda":
        raise NotImplementedError("router_softmax_topk6_triton requires CUDA tensors")
    if logits.dtype != torch.float32:
        raise NotImplementedError("router_softmax_topk6_triton expects fp32 logits")
    if logits.ndim != 2 or not 6 <= logits.shape[1] <= 64:
        raise NotImplementedError("router_softmax_topk6_triton expects [rows, 6..64] logits")
    if not logits.is_contiguous():
        raise NotImplementedError("router_softmax_topk6_triton requires contiguous logits")
    rows = int(logits.shape[0])
    topk_ids = torch.empty((rows, 6), device=logits.device, dtype=torch.long)
    topk_weights = torch.empty((rows, 6), device=logits.device, dtype=torch.float32)
    ids32 = torch.empty((rows, 6), device=logits.device, dtype=torch.int32)
    ops.softmax_topk(logits, float(scaling), topk_ids, ids32, topk_weights)
    return topk_ids, topk_weights
