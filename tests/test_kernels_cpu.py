"""Host-side behaviour of the reference-named drop-in modules (dsv2.kernels.*): load-time
packing layouts and the reference's validation / exception types.  No GPU needed: every
case here raises before any kernel is launched, or only packs weights."""
import types

import pytest
import torch

from dsv2.kernels import (attention_decode_batch, attention_decode_small, attention_prepost, mlp_elementwise,
                          moe_batch, moe_router, moe_small_gemv, rmsnorm)


def test_non_cuda_inputs_raise_not_implemented():
    x = torch.zeros(2, 1, 2048, dtype=torch.bfloat16)
    with pytest.raises(NotImplementedError):
        rmsnorm.rmsnorm_triton(x, torch.ones(2048, dtype=torch.bfloat16), 1e-6)
    with pytest.raises(NotImplementedError):
        mlp_elementwise.silu_mul_triton(x, x)
    with pytest.raises(NotImplementedError):
        attention_prepost.residual_add_triton(x, x)
    with pytest.raises(NotImplementedError):
        moe_router.router_softmax_topk6_triton(torch.zeros(1, 64), 1.0)
    with pytest.raises(NotImplementedError):
        attention_prepost.copy_single_token_to_cache(torch.zeros(1, 16, 1, 8), torch.zeros(1, 16, 4, 8),
                                                     torch.zeros(1, dtype=torch.long))
    packed = moe_batch.PackedRoutedExperts(torch.zeros(2, 128, 64), torch.zeros(2, 64, 64), 64, 64, 2, 6)
    with pytest.raises(NotImplementedError):
        moe_batch.packed_routed_moe(torch.zeros(1, 64), torch.zeros(1, 6, dtype=torch.long), torch.zeros(1, 6),
                                    packed)
    with pytest.raises(NotImplementedError):
        attention_decode_batch.attention_decode_triton(x, None, None, None, None, None, None, None, 0.1)


def test_shape_errors_raise_value_error():
    packed = moe_small_gemv.PackedRoutedExperts(torch.zeros(2, 128, 64), torch.zeros(2, 64, 64), 64, 64, 2, 6)
    with pytest.raises(ValueError):
        moe_small_gemv.batched_grouped_routed_moe_route_gemv(torch.zeros(3, 64), torch.zeros(3, 5, dtype=torch.long),
                                                             torch.zeros(3, 5), packed)
    with pytest.raises(NotImplementedError):   # single-token entry point given 3 rows
        moe_small_gemv.grouped_routed_moe(torch.zeros(3, 64), torch.zeros(3, 6, dtype=torch.long),
                                          torch.zeros(3, 6), packed)


def _expert_list(E, I, H, g):
    def lin(o, i):
        return types.SimpleNamespace(weight=torch.randn(o, i, generator=g))
    return [types.SimpleNamespace(gate_proj=lin(I, H), up_proj=lin(I, H), down_proj=lin(H, I)) for _ in range(E)]


def test_pack_routed_experts_both_module_layouts():
    g = torch.Generator().manual_seed(0)
    E, I, H = 3, 8, 16
    experts = _expert_list(E, I, H, g)
    moe = types.SimpleNamespace(experts=experts, num_experts_per_tok=6, ep_size=1)
    p = moe_batch.pack_routed_experts(moe)
    assert (p.num_experts, p.intermediate_size, p.hidden_size, p.topk) == (E, I, H, 6)
    for e in range(E):
        assert torch.equal(p.gate_up_weights[e, :I], experts[e].gate_proj.weight)
        assert torch.equal(p.gate_up_weights[e, I:], experts[e].up_proj.weight)
        assert torch.equal(p.down_weights[e], experts[e].down_proj.weight)
    # transformers' native 3-D experts: already [E, 2I, H] (gate rows first) / [E, H, I]
    native = types.SimpleNamespace(gate_up_proj=torch.nn.Parameter(p.gate_up_weights.clone()),
                                   down_proj=torch.nn.Parameter(p.down_weights.clone()))
    moe2 = types.SimpleNamespace(experts=native, config=types.SimpleNamespace(num_experts_per_tok=6))
    p2 = moe_small_gemv.pack_routed_experts(moe2)
    assert torch.equal(p2.gate_up_weights, p.gate_up_weights) and torch.equal(p2.down_weights, p.down_weights)
    assert (p2.num_experts, p2.intermediate_size, p2.hidden_size, p2.topk) == (E, I, H, 6)
    with pytest.raises(NotImplementedError):
        moe_batch.pack_routed_experts(types.SimpleNamespace(experts=experts, ep_size=2))


def test_pack_attention_weights_layout():
    g = torch.Generator().manual_seed(1)

    def lin(o, i):
        return types.SimpleNamespace(weight=torch.randn(o, i, generator=g), bias=None)

    attn = types.SimpleNamespace(q_proj=lin(3072, 2048), kv_a_proj_with_mqa=lin(576, 2048), kv_b_proj=lin(4096, 512),
                                 o_proj=lin(2048, 2048),
                                 kv_a_layernorm=types.SimpleNamespace(weight=torch.ones(512), variance_epsilon=1e-6))
    p = attention_decode_small.pack_attention_weights(attn)
    assert p.q_kv_a_weight.shape == (3648, 2048)
    assert torch.equal(p.q_kv_a_weight[:3072], attn.q_proj.weight)
    assert torch.equal(p.q_kv_a_weight[3072:], attn.kv_a_proj_with_mqa.weight)
    assert p.kv_a_ln_eps == 1e-6
    # absorbed W_UK^T: w_uk_t[h, c, d] = kv_b[h * 256 + d, c]
    h, c, d = 5, 300, 77
    assert p.w_uk_t.shape == (16, 512, 128)
    assert p.w_uk_t[h, c, d] == attn.kv_b_proj.weight[h * 256 + d, c]
    attn.q_proj = lin(3000, 2048)
    with pytest.raises(NotImplementedError):
        attention_decode_batch.pack_attention_weights(attn)


def test_run_cli_arguments():
    from dsv2 import run
    a = run._parse_args(["--batch-sizes", "1, 32 256", "--kernel-family", "batch"])
    assert run._batch_sizes(a) == [1, 32, 256] and a.kernel_family == "batch"
    assert run._batch_sizes(run._parse_args(["--batch-size", "4"])) == [4]
    with pytest.raises(ValueError):
        run._batch_sizes(run._parse_args(["--batch-sizes", "0"]))
    if not torch.cuda.is_available():
        with pytest.raises(RuntimeError):
            run.main(["--layers", "1"])


def test_torch_custom_ops_registered():
    import dsv2.torch_ops  # noqa: F401  (registers torch.ops.dsv2.*)
    for name in ("rmsnorm", "silu_mul", "residual_add", "copy_single_token_to_cache", "prepare_decode_inputs",
                 "router_softmax_topk6", "routed_moe", "attention_decode"):
        assert hasattr(torch.ops.dsv2, name), name
    from torch._subclasses.fake_tensor import FakeTensorMode
    with FakeTensorMode():
        x = torch.empty(3, 1, 2048, dtype=torch.bfloat16)
        y = torch.ops.dsv2.rmsnorm(x, torch.empty(2048, dtype=torch.bfloat16), 1e-6)
        assert y.shape == x.shape and y.dtype == x.dtype
        ids, w = torch.ops.dsv2.router_softmax_topk6(torch.empty(5, 64), 1.0)
        assert ids.shape == (5, 6) and ids.dtype == torch.long and w.dtype == torch.float32
    with pytest.raises(NotImplementedError):   # real implementation: CUDA only
        torch.ops.dsv2.rmsnorm(torch.zeros(2, 2048, dtype=torch.bfloat16), torch.ones(2048), 1e-6)
