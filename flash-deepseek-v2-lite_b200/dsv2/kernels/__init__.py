"""Drop-in replacements for the reference's ``triton_kernels`` package.

Each module carries the name of the reference module it replaces and exports the same
functions and dataclasses (names, argument meaning, return values, exception types),
so a caller written against ``triton_kernels.X`` only changes its import to
``dsv2.kernels.X``:

  rmsnorm                 rmsnorm_triton
  mlp_elementwise         silu_mul_triton
  attention_prepost       copy_single_token_to_cache, prepare_decode_inputs_triton,
                          residual_add_triton
  moe_router              router_softmax_topk6_triton
  moe_batch               PackedRoutedExperts, pack_routed_experts, packed_routed_moe,
                          batched_grouped_routed_moe
  moe_small_gemv          PackedRoutedExperts, pack_routed_experts, grouped_routed_moe,
                          batched_grouped_routed_moe_route_gemv
  attention_decode_small  AttentionPackedWeights, pack_attention_weights,
                          attention_decode_only_triton, attention_decode_small_batch_triton
  attention_decode_batch  AttentionPackedWeights, pack_attention_weights,
                          attention_decode_triton

All compute runs in libdsv2.so (sm_100a kernels); there is no Triton and no CPU path
(the reference's eager torch fallbacks, e.g. packed_routed_moe_eager, are not provided:
a non-CUDA input raises NotImplementedError).
Outputs are allocated with the torch caching allocator (as the reference does), or are
persistent per-(device, batch) workspaces owned by the packed weights (attention), so
the calls can be captured in a CUDA graph after one warm-up call.

The attention functions take the 576-wide latent cache in ``key_cache`` ([B, S, 576]
bf16: RMS-normalised latent ++ roped k_pe) and ignore ``value_cache``; the expanded
per-head K/V cache of the reference has no counterpart (absorbed MLA never builds it).
"""
