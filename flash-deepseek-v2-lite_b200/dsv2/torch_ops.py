"""The drop-in kernels registered as torch custom operators (``torch.ops.dsv2.*``).

Importing this module registers, over the same libdsv2 entry points as dsv2.kernels:

  torch.ops.dsv2.rmsnorm(hidden_states, weight, eps) -> Tensor
  torch.ops.dsv2.silu_mul(gate, up) -> Tensor
  torch.ops.dsv2.residual_add(a, b) -> Tensor
  torch.ops.dsv2.copy_single_token_to_cache(src, dst!, cache_position) -> ()
  torch.ops.dsv2.prepare_decode_inputs(cache_position, attention_mask!, position_ids!,
                                       attention_mask_index) -> ()
  torch.ops.dsv2.router_softmax_topk6(logits, scaling) -> (Tensor ids, Tensor weights)
  torch.ops.dsv2.routed_moe(x, topk_ids, topk_weight, gate_up_weights, down_weights,
                            family) -> Tensor          family 0 = small (GEMV), 1 = batch
  torch.ops.dsv2.attention_decode(hidden_states, cos, sin, position_ids, cache_position,
                                  key_cache!, q_kv_a_weight, kv_b_weight, o_weight, w_uk_t,
                                  kv_a_ln_weight, kv_a_ln_eps, softmax_scale, family) -> Tensor

(``!`` = mutated in place).  The operators take tensors and scalars only, so the
packed-weight objects of the Python API are passed as their tensors.  Each operator
has a fake (meta) implementation for tracing; the real one runs the CUDA kernels and
raises like the Python API on unsupported inputs.
"""
from __future__ import annotations

import torch

from .kernels import attention_prepost, mlp_elementwise, moe_router, rmsnorm
from .kernels._attention import AttentionPackedWeights, mla_decode_layer
from .kernels._moe import PackedRoutedExperts, routed_moe as _routed_moe

_lib = torch.library


@_lib.custom_op("dsv2::rmsnorm", mutates_args=())
def rmsnorm_op(hidden_states: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    return rmsnorm.rmsnorm_triton(hidden_states, weight, eps)


@rmsnorm_op.register_fake
def _(hidden_states, weight, eps):
    return torch.empty_like(hidden_states)


@_lib.custom_op("dsv2::silu_mul", mutates_args=())
def silu_mul_op(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    return mlp_elementwise.silu_mul_triton(gate, up)


@silu_mul_op.register_fake
def _(gate, up):
    return torch.empty_like(gate)


@_lib.custom_op("dsv2::residual_add", mutates_args=())
def residual_add_op(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    return attention_prepost.residual_add_triton(a, b)


@residual_add_op.register_fake
def _(a, b):
    return torch.empty_like(a)


@_lib.custom_op("dsv2::copy_single_token_to_cache", mutates_args=("dst",))
def copy_single_token_to_cache_op(src: torch.Tensor, dst: torch.Tensor, cache_position: torch.Tensor) -> None:
    attention_prepost.copy_single_token_to_cache(src, dst, cache_position)


@copy_single_token_to_cache_op.register_fake
def _(src, dst, cache_position):
    return None


@_lib.custom_op("dsv2::prepare_decode_inputs", mutates_args=("attention_mask", "position_ids"))
def prepare_decode_inputs_op(cache_position: torch.Tensor, attention_mask: torch.Tensor,
                             position_ids: torch.Tensor, attention_mask_index: torch.Tensor) -> None:
    attention_prepost.prepare_decode_inputs_triton(cache_position, attention_mask, position_ids,
                                                   attention_mask_index)


@prepare_decode_inputs_op.register_fake
def _(cache_position, attention_mask, position_ids, attention_mask_index):
    return None


@_lib.custom_op("dsv2::router_softmax_topk6", mutates_args=())
def router_softmax_topk6_op(logits: torch.Tensor, scaling: float) -> tuple[torch.Tensor, torch.Tensor]:
    return moe_router.router_softmax_topk6_triton(logits, scaling)


@router_softmax_topk6_op.register_fake
def _(logits, scaling):
    rows = logits.shape[0]
    return (logits.new_empty((rows, 6), dtype=torch.long), logits.new_empty((rows, 6), dtype=torch.float32))


@_lib.custom_op("dsv2::routed_moe", mutates_args=())
def routed_moe_op(x: torch.Tensor, topk_ids: torch.Tensor, topk_weight: torch.Tensor,
                  gate_up_weights: torch.Tensor, down_weights: torch.Tensor, family: int) -> torch.Tensor:
    E, two_i, H = gate_up_weights.shape
    packed = PackedRoutedExperts(gate_up_weights=gate_up_weights, down_weights=down_weights, hidden_size=H,
                                 intermediate_size=two_i // 2, num_experts=E, topk=int(topk_ids.shape[1]))
    return _routed_moe("routed_moe", x, topk_ids, topk_weight, packed, None, int(family))


@routed_moe_op.register_fake
def _(x, topk_ids, topk_weight, gate_up_weights, down_weights, family):
    return torch.empty_like(x)


@_lib.custom_op("dsv2::attention_decode", mutates_args=("key_cache",))
def attention_decode_op(hidden_states: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                        position_ids: torch.Tensor, cache_position: torch.Tensor, key_cache: torch.Tensor,
                        q_kv_a_weight: torch.Tensor, kv_b_weight: torch.Tensor, o_weight: torch.Tensor,
                        w_uk_t: torch.Tensor, kv_a_ln_weight: torch.Tensor, kv_a_ln_eps: float,
                        softmax_scale: float, family: int) -> torch.Tensor:
    key = (q_kv_a_weight.data_ptr(), kv_b_weight.data_ptr(), o_weight.data_ptr())
    packed = _PACKED.get(key)
    if packed is None:
        packed = AttentionPackedWeights(q_kv_a_weight=q_kv_a_weight, kv_b_weight=kv_b_weight, o_weight=o_weight,
                                        kv_a_ln_weight=kv_a_ln_weight, kv_a_ln_eps=float(kv_a_ln_eps),
                                        w_uk_t=w_uk_t)
        _PACKED[key] = packed
    out = mla_decode_layer("attention_decode", hidden_states, cos, sin, position_ids, cache_position, key_cache,
                           None, packed, softmax_scale, int(family), single_row=False)
    return out.clone()


@attention_decode_op.register_fake
def _(hidden_states, cos, sin, position_ids, cache_position, key_cache, q_kv_a_weight, kv_b_weight, o_weight,
      w_uk_t, kv_a_ln_weight, kv_a_ln_eps, softmax_scale, family):
    return torch.empty_like(hidden_states)


# per-weight-set workspaces of the attention operator (keyed by the weights' addresses)
_PACKED: dict = {}
