"""Routed-expert packing and the grouped MoE shared by moe_batch and moe_small_gemv.

Reference: PackedRoutedExperts / pack_routed_experts (moe_batch.py:12-30, :324-363, the
same in moe_small_gemv.py:11-27, :364-403) and the routed MoE they feed.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .. import ops

_SLOTS = 8   # per-token slots of the fp32 partial buffer (route_slot = token * 8 + k)


@dataclass
class PackedRoutedExperts:
    # gate_up_weights: [num_experts, 2 * intermediate_size, hidden_size] (gate rows, then up rows)
    # down_weights:    [num_experts, hidden_size, intermediate_size]
    gate_up_weights: torch.Tensor
    down_weights: torch.Tensor
    hidden_size: int
    intermediate_size: int
    num_experts: int
    topk: int

    def to(self, *args, **kwargs) -> "PackedRoutedExperts":
        self.gate_up_weights = self.gate_up_weights.to(*args, **kwargs)
        self.down_weights = self.down_weights.to(*args, **kwargs)
        return self


def pack_routed_experts(moe: torch.nn.Module, device: torch.device | str | None = None) -> PackedRoutedExperts:
    """Stack the routed experts of an MoE block into the packed layout.

    Accepts the per-expert module list of the checkpoint's modeling code
    (moe.experts[i].gate_proj / up_proj / down_proj, as the reference reads) and the 3-D
    parameters of transformers' native DeepseekV2Experts (experts.gate_up_proj
    [E, 2I, H] with gate rows first, experts.down_proj [E, H, I]), which already are
    this layout."""
    if getattr(moe, "ep_size", 1) != 1:
        raise NotImplementedError("pack_routed_experts currently only supports ep_size == 1")
    topk = int(getattr(moe, "num_experts_per_tok", 0) or getattr(getattr(moe, "config", None),
                                                                   "num_experts_per_tok", 0) or 6)
    ex = moe.experts
    if hasattr(ex, "gate_up_proj"):
        gate_up = ex.gate_up_proj.data
        down = ex.down_proj.data
        if device is not None:
            gate_up, down = gate_up.to(device), down.to(device)
        gate_up, down = gate_up.contiguous(), down.contiguous()
        num_experts, two_i, hidden = (int(s) for s in gate_up.shape)
        inter = two_i // 2
    else:
        experts = [e for e in ex if e is not None]
        if not experts:
            raise ValueError("No local routed experts found to pack")
        first = experts[0].gate_proj.weight
        dev = first.device if device is None else device
        inter, hidden = (int(s) for s in first.shape)
        num_experts = len(experts)
        gate_up = torch.empty((num_experts, 2 * inter, hidden), device=dev, dtype=first.dtype)
        down = torch.empty((num_experts, hidden, inter), device=dev, dtype=first.dtype)
        for i, e in enumerate(experts):
            gate_up[i, :inter].copy_(e.gate_proj.weight)
            gate_up[i, inter:].copy_(e.up_proj.weight)
            down[i].copy_(e.down_proj.weight)
    return PackedRoutedExperts(gate_up_weights=gate_up, down_weights=down, hidden_size=hidden,
                               intermediate_size=inter, num_experts=num_experts, topk=topk)


def _check(name: str, x: torch.Tensor, topk_ids: torch.Tensor, topk_weight: torch.Tensor,
           packed: PackedRoutedExperts, output_dtype) -> torch.dtype:
    if x.ndim != 2 or topk_ids.ndim != 2 or topk_weight.ndim != 2:
        raise ValueError(f"{name} expects x=[B,H], topk tensors=[B,topk]")
    if topk_ids.shape != topk_weight.shape or topk_ids.shape[0] != x.shape[0]:
        raise ValueError("topk_ids/topk_weight must have shape [B, topk]")
    if topk_ids.shape[1] != packed.topk:
        raise ValueError(f"Expected topk={packed.topk}, got {topk_ids.shape[1]}")
    if x.device.type != "cuda":
        raise NotImplementedError(f"{name} requires CUDA")
    if packed.topk != 6:
        raise NotImplementedError(f"{name} currently supports topk=6, got {packed.topk}")
    if x.dtype != torch.bfloat16 or packed.gate_up_weights.dtype != torch.bfloat16 \
            or packed.down_weights.dtype != torch.bfloat16:
        raise NotImplementedError(f"{name} supports bf16 activations and weights")
    if x.shape[1] != packed.hidden_size or packed.hidden_size % 64 or packed.intermediate_size % 64:
        raise NotImplementedError(f"{name}: hidden/intermediate sizes must be multiples of 64")
    if packed.num_experts > 64 or x.shape[0] > 4096:
        raise NotImplementedError(f"{name}: at most 64 experts and 4096 rows")
    if output_dtype is None:
        output_dtype = x.dtype
    if output_dtype not in (torch.bfloat16, torch.float32):
        raise NotImplementedError(f"{name}: output dtype must be bf16 or fp32")
    if packed.gate_up_weights.device != x.device or packed.down_weights.device != x.device:
        packed.to(device=x.device)
    return output_dtype


def routed_moe(name: str, x: torch.Tensor, topk_ids: torch.Tensor, topk_weight: torch.Tensor,
               packed: PackedRoutedExperts, output_dtype, family: int) -> torch.Tensor:
    """out[b] = sum_k w[b,k] * down_e(silu(gate_e(x[b])) * up_e(x[b])), e = ids[b,k].

    Launches: bucket routes by expert (stable, + expert-ordered copy of x for the
    batch family) -> grouped gate_up GEMM with the SwiGLU epilogue and grouped down GEMM
    scaling each route by its weight into per-slot fp32 partials (batch family: one fused
    tcgen05 launch; small family: two mma.sync GEMV launches) -> fixed-order sum of the
    six slots."""
    out_dtype = _check(name, x, topk_ids, topk_weight, packed, output_dtype)
    x = x.contiguous()
    B, H = (int(s) for s in x.shape)
    E, I, K = packed.num_experts, packed.intermediate_size, packed.topk
    dev = x.device
    R = B * K
    out = torch.empty((B, H), device=dev, dtype=out_dtype)
    if B == 0:
        return out
    ids32 = topk_ids.to(torch.int32).contiguous()
    tw = topk_weight.to(torch.float32).contiguous()
    go = torch.empty(E + 3, device=dev, dtype=torch.int32)   # E experts + two (empty) shared groups
    rt = torch.empty(R, device=dev, dtype=torch.int32)
    rs = torch.empty(R, device=dev, dtype=torch.int32)
    rw = torch.empty(R, device=dev, dtype=torch.float32)
    h = torch.empty((R, I), device=dev, dtype=torch.bfloat16)
    partial = torch.empty((B, _SLOTS, H), device=dev, dtype=torch.float32)
    batch = family == ops.FAMILY_BATCH
    xs = torch.empty((R, H), device=dev, dtype=torch.bfloat16) if batch else None
    ops.moe_bucket(ids32, tw, 0, E, 0, 0, go, rt, rs, rw, gather_src=x if batch else None, gather_out=xs)
    if batch:
        sync = torch.zeros(E + 2, device=dev, dtype=torch.int32)
        ops.moe(gate_up=packed.gate_up_weights, down=packed.down_weights, x_sorted=xs, h=h, group_offsets=go,
                max_routes_per_group=B, route_slot=rs, route_weight=rw, y=partial.view(-1, H), sync=sync)
        ops.sum_partials(partial[:, :K], out)
        return out
    ops.linear(w=packed.gate_up_weights, n_rows=I, k=H, up_offset=I * H, w_group_stride=2 * I * H,
               x=xs if batch else x, y=h, epilogue=ops.EPI_SWIGLU, n_groups=E, group_offsets=go,
               max_routes_per_group=B, route_x_row=None if batch else rt, family=family,
               w_group_rows=2 * I, x_group_rows=R if batch else B)
    ops.linear(w=packed.down_weights, n_rows=H, k=I, w_group_stride=H * I, x=h, y=partial.view(-1, H),
               epilogue=ops.EPI_SCALE_F32, n_groups=E, group_offsets=go, max_routes_per_group=B,
               route_y_row=rs, route_scale=rw, family=family, w_group_rows=H, x_group_rows=R,
               offsets_prior=True)
    ops.sum_partials(partial[:, :K], out)
    return out
