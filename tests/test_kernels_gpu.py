"""GPU parity of the reference-named drop-in modules (dsv2.kernels.*) against the oracle
(oracle/ops.py) and the reference kernels' golden outputs (tests/golden/).

Tolerances: elementwise/norm outputs to 1 bf16 ulp; the MoE and attention pipelines,
whose GEMM accumulation order differs from the oracle's, to max|err| / max|ref| <= 2e-2
(bf16 intermediates, as in the model's own forward).
"""
import math
import types

import pytest
import torch

from oracle import ops as O

pytestmark = pytest.mark.gpu

DEV = "cuda"


def relerr(a, b):
    a, b = a.double().cpu(), b.double().cpu()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))


@pytest.fixture(scope="module")
def K():
    from dsv2._lib import load
    load()
    from dsv2.kernels import (attention_decode_batch, attention_decode_small, attention_prepost,
                              mlp_elementwise, moe_batch, moe_router, moe_small_gemv, rmsnorm)
    return types.SimpleNamespace(rmsnorm=rmsnorm, mlp=mlp_elementwise, pre=attention_prepost, router=moe_router,
                                 moe_batch=moe_batch, moe_small=moe_small_gemv, attn_small=attention_decode_small,
                                 attn_batch=attention_decode_batch)


def test_rmsnorm_triton_golden(K, golden_ref):
    for key, shape in (("rmsnorm_2048", (5, 1, 2048)), ("rmsnorm_512", (3, 512))):
        g = golden_ref[key]
        x = g["x"].reshape(shape).to(DEV)
        y = K.rmsnorm.rmsnorm_triton(x, g["w"].to(DEV), g["eps"])
        assert y.shape == x.shape and y.dtype == x.dtype
        torch.testing.assert_close(y.reshape(g["y"].shape).cpu().float(), g["y"].float(), rtol=2 ** -7, atol=1e-6)


@pytest.mark.parametrize("wdt", [torch.float16, torch.float32, torch.bfloat16])
def test_rmsnorm_and_residual_add_fp16(K, wdt):
    """fp16 activations, as the reference's wrappers accept (rmsnorm.py:64-65,
    attention_prepost.py:197-198): within one fp16 rounding of the oracle's fp32 math."""
    g = torch.Generator().manual_seed(17)
    x = torch.randn(6, 1, 2048, generator=g).to(torch.float16)
    w = (1 + 0.1 * torch.randn(2048, generator=g)).to(wdt)
    y = K.rmsnorm.rmsnorm_triton(x.to(DEV), w.to(DEV), 1e-6)
    assert y.dtype == torch.float16 and y.shape == x.shape
    torch.testing.assert_close(y.cpu().float(), O.rmsnorm(x, w, 1e-6).float(), rtol=2 ** -10, atol=1e-5)
    a = torch.randn(4, 1, 2048, generator=g).to(torch.float16)
    b = torch.randn(4, 1, 2048, generator=g).to(torch.float16)
    out = K.pre.residual_add_triton(a.to(DEV), b.to(DEV))
    assert out.dtype == torch.float16
    assert torch.equal(out.cpu(), O.residual_add(a, b))
    with pytest.raises(NotImplementedError):
        K.pre.residual_add_triton(a.to(DEV), b.to(DEV).to(torch.bfloat16))


def test_elementwise_golden(K, golden_ref):
    g = golden_ref["residual_add"]
    out = K.pre.residual_add_triton(g["a"].to(DEV), g["b"].to(DEV))
    assert torch.equal(out.cpu(), O.residual_add(g["a"], g["b"]))
    torch.testing.assert_close(out.cpu().float(), g["out"].float(), rtol=2 ** -7, atol=0)
    g = golden_ref["silu_mul"]
    out = K.mlp.silu_mul_triton(g["gate"].to(DEV), g["up"].to(DEV))
    torch.testing.assert_close(out.cpu().float(), g["out"].float(), rtol=2 ** -7, atol=1e-6)
    with pytest.raises(ValueError):
        K.mlp.silu_mul_triton(g["gate"].to(DEV), g["up"].to(DEV)[:2])


def test_prepare_inputs_and_cache_copy_golden(K, golden_ref):
    g = golden_ref["prepare_decode_inputs"]
    B, S = g["batch"], g["attention_mask_index"].numel()
    mask = torch.empty(B, S, dtype=torch.int64, device=DEV)
    pid = torch.empty(B, 1, dtype=torch.int64, device=DEV)
    K.pre.prepare_decode_inputs_triton(g["cache_position"].to(DEV), mask, pid, g["attention_mask_index"].to(DEV))
    assert torch.equal(mask.cpu(), g["attention_mask"]) and torch.equal(pid.cpu(), g["position_ids"])
    with pytest.raises(ValueError):
        K.pre.prepare_decode_inputs_triton(g["cache_position"].to(DEV), mask[:, :5], pid,
                                           g["attention_mask_index"].to(DEV))
    g = golden_ref["copy_single_token_to_cache"]
    dst = g["dst_before"].to(DEV)
    K.pre.copy_single_token_to_cache(g["src"].to(DEV), dst, g["cache_position"].to(DEV))
    assert torch.equal(dst.cpu(), g["dst_after"])


def test_router_softmax_topk6_golden(K, golden_ref):
    g = golden_ref["router_topk6"]
    ids, w = K.router.router_softmax_topk6_triton(g["logits"].to(DEV), g["scaling"])
    assert ids.dtype == torch.int64 and w.dtype == torch.float32
    assert torch.equal(ids.cpu(), g["ids"])
    torch.testing.assert_close(w.cpu(), g["weights"], rtol=1e-5, atol=1e-7)
    ids1, w1 = K.router.router_softmax_topk6_triton(g["logits"][:1].contiguous().to(DEV), 2.5)
    oi, ow = O.softmax_topk6(g["logits"][:1], 2.5)
    assert torch.equal(ids1.cpu(), oi)
    torch.testing.assert_close(w1.cpu(), ow, rtol=1e-5, atol=1e-7)
    with pytest.raises(NotImplementedError):
        K.router.router_softmax_topk6_triton(g["logits"].to(DEV).double(), 1.0)


# ---------------------------------------------------------------------------- MoE
E, H, I = 16, 2048, 1408


@pytest.fixture(scope="module")
def experts():
    g = torch.Generator().manual_seed(11)
    gate_up = (torch.randn(E, 2 * I, H, generator=g) * 0.02).to(torch.bfloat16)
    down = (torch.randn(E, H, I, generator=g) * 0.02).to(torch.bfloat16)
    return gate_up, down


def _moe_case(B, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(B, H, generator=g).to(torch.bfloat16)
    ids = torch.stack([torch.randperm(E, generator=g)[:6] for _ in range(B)])
    w = torch.rand(B, 6, generator=g)
    return x, ids, w


def _moe_oracle(x, ids, w, gate_up, down):
    out = torch.zeros(x.shape[0], H)
    for b in range(x.shape[0]):
        for k in range(6):
            e = int(ids[b, k])
            out[b] += O.expert_mlp(x[b:b + 1], gate_up[e], down[e])[0].float() * float(w[b, k])
    return out


@pytest.mark.parametrize("fn,B", [("grouped_routed_moe", 1), ("batched_grouped_routed_moe_route_gemv", 5),
                                  ("packed_routed_moe", 1), ("packed_routed_moe", 37),
                                  ("batched_grouped_routed_moe", 128)])
def test_routed_moe_vs_oracle(K, experts, fn, B):
    gate_up, down = experts
    mod = K.moe_batch if fn in ("packed_routed_moe", "batched_grouped_routed_moe") else K.moe_small
    packed = mod.PackedRoutedExperts(gate_up_weights=gate_up.to(DEV), down_weights=down.to(DEV), hidden_size=H,
                                     intermediate_size=I, num_experts=E, topk=6)
    x, ids, w = _moe_case(B, seed=B)
    y = getattr(mod, fn)(x.to(DEV), ids.to(DEV), w.to(DEV), packed)
    assert y.shape == (B, H) and y.dtype == torch.bfloat16
    ref = _moe_oracle(x, ids, w, gate_up, down)
    assert relerr(y, ref) < 2e-2
    y32 = getattr(mod, fn)(x.to(DEV), ids.to(DEV), w.to(DEV), packed, output_dtype=torch.float32)
    assert y32.dtype == torch.float32
    assert relerr(y32, ref) < 2e-2
    torch.testing.assert_close(y32.to(torch.bfloat16).cpu().float(), y.cpu().float(), rtol=2 ** -7, atol=0)


def test_routed_moe_errors(K, experts):
    gate_up, down = experts
    packed = K.moe_batch.PackedRoutedExperts(gate_up_weights=gate_up[:2].to(DEV), down_weights=down[:2].to(DEV),
                                             hidden_size=H, intermediate_size=I, num_experts=2, topk=6)
    x = torch.zeros(3, H, dtype=torch.bfloat16, device=DEV)
    ids = torch.zeros(3, 5, dtype=torch.int64, device=DEV)
    with pytest.raises(ValueError):
        K.moe_batch.packed_routed_moe(x, ids, torch.zeros(3, 5, device=DEV), packed)
    with pytest.raises(NotImplementedError):
        K.moe_small.grouped_routed_moe(x, torch.zeros(3, 6, dtype=torch.int64, device=DEV),
                                       torch.zeros(3, 6, device=DEV), packed)


# ---------------------------------------------------------------------- attention
def _attn_module(seed):
    g = torch.Generator().manual_seed(seed)

    def lin(o, i, s=0.02):
        return types.SimpleNamespace(weight=(torch.randn(o, i, generator=g) * s).to(torch.bfloat16), bias=None)

    return types.SimpleNamespace(
        q_proj=lin(3072, 2048), kv_a_proj_with_mqa=lin(576, 2048), kv_b_proj=lin(4096, 512, 0.05),
        o_proj=lin(2048, 2048),
        kv_a_layernorm=types.SimpleNamespace(weight=(1 + 0.1 * torch.randn(512, generator=g)).to(torch.bfloat16),
                                             variance_epsilon=1e-6))


def _to_dev(attn):
    def cp(ns):
        return types.SimpleNamespace(**{k: (v.to(DEV) if torch.is_tensor(v) else v) for k, v in vars(ns).items()})
    return types.SimpleNamespace(**{k: cp(v) for k, v in vars(attn).items()})


def _rope(S):
    inv = 1.0 / (10000.0 ** (torch.arange(0, 64, 2, dtype=torch.float32) / 64))
    f = torch.arange(S, dtype=torch.float32)[:, None] * inv[None, :]
    cos32, sin32 = torch.cos(f), torch.sin(f)
    # reference layout: [S, 64] = the 32 angles twice (the HF rotary cache)
    return cos32, sin32, torch.cat([cos32, cos32], 1), torch.cat([sin32, sin32], 1)


@pytest.mark.parametrize("fn,B,ragged", [("attention_decode_only_triton", 1, False),
                                         ("attention_decode_small_batch_triton", 4, True),
                                         ("attention_decode_triton", 4, False),
                                         ("attention_decode_triton", 64, True)])
def test_attention_decode_vs_oracle(K, fn, B, ragged):
    S = 160
    attn = _attn_module(seed=B)
    mod = K.attn_batch if fn == "attention_decode_triton" else K.attn_small
    packed = mod.pack_attention_weights(_to_dev(attn))
    g = torch.Generator().manual_seed(100 + B)
    x = torch.randn(B, 1, 2048, generator=g).to(torch.bfloat16)
    if ragged:
        pos = torch.randint(0, S, (B,), generator=g)
    else:
        pos = torch.full((B,), 97)
    cache = torch.randn(B, S, 576, generator=g).to(torch.bfloat16)
    cos32, sin32, cos64, sin64 = _rope(S)
    scale = 192 ** -0.5
    cache_d = cache.to(DEV)
    cp = (pos if ragged else pos[:1]).to(DEV)
    y = getattr(mod, fn)(x.to(DEV), cos64.to(DEV), sin64.to(DEV), pos.view(B, 1).to(DEV), cp, cache_d, None,
                         packed, scale)
    assert y.shape == (B, 1, 2048) and y.dtype == torch.bfloat16
    cache_o = cache.clone()
    ref = O.absorbed_attention_layer(x.view(B, 2048), attn, cache_o, pos, cos32, sin32, scale)
    assert relerr(y.view(B, 2048), ref) < 2e-2
    rows = cache_d.cpu()[torch.arange(B), pos]
    assert relerr(rows, cache_o[torch.arange(B), pos]) < 2e-2
    # only the new position of each row is written
    keep = torch.ones(B, S, dtype=torch.bool)
    keep[torch.arange(B), pos] = False
    assert torch.equal(cache_d.cpu()[keep], cache[keep])


def test_attention_small_and_batch_families_agree(K):
    B, S = 8, 96
    attn = _to_dev(_attn_module(seed=7))
    ps = K.attn_small.pack_attention_weights(attn)
    pb = K.attn_batch.pack_attention_weights(attn)
    g = torch.Generator().manual_seed(5)
    x = torch.randn(B, 1, 2048, generator=g).to(torch.bfloat16).to(DEV)
    cache = torch.randn(B, S, 576, generator=g).to(torch.bfloat16).to(DEV)
    pos = torch.randint(1, S, (B,), generator=g).to(DEV)
    _, _, cos64, sin64 = _rope(S)
    c1, c2 = cache.clone(), cache.clone()
    ys = K.attn_small.attention_decode_small_batch_triton(x, cos64.to(DEV), sin64.to(DEV), pos.view(B, 1), pos, c1,
                                                          None, ps, 0.07).clone()
    yb = K.attn_batch.attention_decode_triton(x, cos64.to(DEV), sin64.to(DEV), pos.view(B, 1), pos, c2, None, pb,
                                              0.07)
    assert relerr(ys, yb) < 2e-2
    with pytest.raises(ValueError):
        K.attn_batch.attention_decode_triton(x, cos64.to(DEV), sin64.to(DEV), pos.view(1, B), pos, c2, None, pb, 0.07)


def test_run_cli_json(capsys):
    import json

    from dsv2 import run
    run.main(["--layers", "2", "--prompt-len", "16", "--max-new-tokens", "5", "--batch-sizes", "1 3",
              "--dump-token-ids", "--dump-step-trace"])
    doc = json.loads(capsys.readouterr().out)
    r1, r3 = doc["results"]
    assert r1["batch_size"] == 1 and r1["path"] == "dsv2_small_graph" and r1["decode_tokens"] == 4
    assert r3["batch_size"] == 3 and r3["decode_tokens"] == 12 and r1["tps"] > 0 and r1["ttft_ms"] > 0
    assert len(r1["generated_token_ids"]) == 5 and len(r3["generated_token_ids"]) == 3
    # one prompt replicated over the batch: every row decodes the same greedy tokens
    assert all(row == r3["generated_token_ids"][0] for row in r3["generated_token_ids"])
    assert [e["step"] for e in r1["step_trace"]] == list(range(5))
    assert r1["step_trace"][1]["cache_position"] == 17
    assert doc["hardware"]["gpu"]["capability"] == "sm100"


def test_torch_ops_match_python_api(K, experts):
    """torch.ops.dsv2.* (custom operators) return what the reference-named functions return."""
    import dsv2.torch_ops  # noqa: F401
    gate_up, down = experts
    gud, dnd = gate_up.to(DEV), down.to(DEV)
    x, ids, w = _moe_case(9, seed=9)
    packed = K.moe_batch.PackedRoutedExperts(gate_up_weights=gud, down_weights=dnd, hidden_size=H,
                                             intermediate_size=I, num_experts=E, topk=6)
    for fam, fn in ((1, K.moe_batch.packed_routed_moe), (0, K.moe_small.batched_grouped_routed_moe_route_gemv)):
        a = fn(x.to(DEV), ids.to(DEV), w.to(DEV), packed)
        b = torch.ops.dsv2.routed_moe(x.to(DEV), ids.to(DEV), w.to(DEV), gud, dnd, fam)
        assert torch.equal(a, b)
    g = torch.Generator().manual_seed(3)
    y = torch.randn(4, 1, 2048, generator=g).to(torch.bfloat16).to(DEV)
    wt = torch.rand(2048, generator=g).to(torch.bfloat16).to(DEV)
    assert torch.equal(torch.ops.dsv2.rmsnorm(y, wt, 1e-6), K.rmsnorm.rmsnorm_triton(y, wt, 1e-6))
    attn = _to_dev(_attn_module(seed=21))
    p = K.attn_batch.pack_attention_weights(attn)
    B, S = 3, 64
    xh = torch.randn(B, 1, 2048, generator=g).to(torch.bfloat16).to(DEV)
    cache = torch.randn(B, S, 576, generator=g).to(torch.bfloat16).to(DEV)
    pos = torch.tensor([5, 30, 63], device=DEV)
    _, _, cos64, sin64 = _rope(S)
    c1, c2 = cache.clone(), cache.clone()
    a = K.attn_batch.attention_decode_triton(xh, cos64.to(DEV), sin64.to(DEV), pos.view(B, 1), pos, c1, None, p,
                                             0.07).clone()
    b = torch.ops.dsv2.attention_decode(xh, cos64.to(DEV), sin64.to(DEV), pos.view(B, 1), pos, c2, p.q_kv_a_weight,
                                        p.kv_b_weight, p.o_weight, p.w_uk_t, p.kv_a_ln_weight, p.kv_a_ln_eps, 0.07, 1)
    assert torch.equal(a, b) and torch.equal(c1, c2)
