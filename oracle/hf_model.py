"""Oracle model: the Hugging Face eager DeepSeek-V2 (transformers 5.5.0) with seeded weights.

TEST INFRASTRUCTURE ONLY.  Imported by tests/, __graft_entry__.smoke() and the
CPU-baseline / reference arms of bench.py as the checker, never by the decode engine.

The reference (Flash-DeepSeeek-V2-Lite) loads DeepSeek-V2-Lite-Chat with the
checkpoint's remote modeling code (src/run.py:719-725), which is not available
here; its in-container stand-in is transformers' native
models/deepseek_v2/modeling_deepseek_v2.py (a third-party dependency, version
5.5.0), run eagerly (eager attention, eager experts loop).

The architecture constants below are written out here, independently of the package
under test, from the reference's hard-coded shapes (triton_kernels/
attention_decode_small.py:12-21: hidden 2048, 16 heads, kv_lora 512, qk_nope 128,
qk_rope 64, v_head 128), the MoE constants its kernels assume (moe_batch.py:324-363:
64 routed experts of intermediate 1408 packed [gate; up]; moe_router.py:8-60: top-6
greedy softmax routing, weights times routed_scaling_factor, no renormalisation) and
the DeepSeek-V2-Lite configuration those shapes come from (27 layers, the first dense
with intermediate 10944, 2 shared experts, vocab 102400, RMSNorm eps 1e-6, YaRN RoPE
with theta 10000, factor 40 over 4096 original positions, beta_fast 32, beta_slow 1,
mscale / mscale_all_dim 0.707).  tests/test_cpu.py checks that the package's synthetic
model builder produces exactly this configuration and these weights.

Weights: N(0, std) for every matrix and embedding, ones for RMSNorm weights, drawn from
one torch.Generator seeded with `seed` in parameter-registration order on the target
device.
"""
from __future__ import annotations

import torch
from transformers import DeepseekV2Config, DeepseekV2ForCausalLM
from transformers.initialization import no_init_weights

# YaRN RoPE parameters of DeepSeek-V2-Lite (HF modeling_deepseek_v2.py rotary embedding
# with rope_type "yarn")
YARN = {
    "rope_type": "yarn",
    "rope_theta": 10000.0,
    "factor": 40.0,
    "original_max_position_embeddings": 4096,
    "beta_fast": 32.0,
    "beta_slow": 1.0,
    "mscale": 0.707,
    "mscale_all_dim": 0.707,
}

# field -> value of the oracle configuration (also the list the CPU test compares)
ARCH = {
    "vocab_size": 102400,
    "hidden_size": 2048,
    "intermediate_size": 10944,
    "moe_intermediate_size": 1408,
    "num_attention_heads": 16,
    "num_key_value_heads": 16,
    "n_shared_experts": 2,
    "n_routed_experts": 64,
    "num_experts_per_tok": 6,
    "routed_scaling_factor": 1.0,
    "topk_method": "greedy",
    "norm_topk_prob": False,
    "q_lora_rank": None,
    "kv_lora_rank": 512,
    "qk_nope_head_dim": 128,
    "qk_rope_head_dim": 64,
    "v_head_dim": 128,
    "first_k_dense_replace": 1,
    "rms_norm_eps": 1e-6,
    "initializer_range": 0.02,
    "tie_word_embeddings": False,
}


def dsv2_lite_config(num_layers: int = 27) -> DeepseekV2Config:
    """DeepSeek-V2-Lite with `num_layers` decoder layers, eager attention and experts."""
    cfg = DeepseekV2Config(num_hidden_layers=num_layers, max_position_embeddings=163840,
                           rope_parameters=dict(YARN), bos_token_id=100000, eos_token_id=100001,
                           pad_token_id=None, **ARCH)
    cfg._attn_implementation = "eager"
    cfg._experts_implementation = "eager"
    return cfg


@torch.no_grad()
def build_model(cfg: DeepseekV2Config, seed: int, device="cpu", dtype=torch.float32,
                std: float | None = None) -> DeepseekV2ForCausalLM:
    """The HF model without HF's own init, filled from one seeded generator."""
    std = cfg.initializer_range if std is None else std
    prev = torch.get_default_dtype()
    torch.set_default_dtype(dtype)
    try:
        with no_init_weights(), torch.device(device):
            model = DeepseekV2ForCausalLM(cfg)
    finally:
        torch.set_default_dtype(prev)
    model.to(device=device, dtype=dtype)
    gen = torch.Generator(device=device).manual_seed(int(seed))
    for name, p in model.named_parameters():
        if name.endswith("norm.weight") or "layernorm" in name:
            p.fill_(1.0)
        else:
            p.normal_(0.0, std, generator=gen)
    model.eval()
    return model


def router_bias_zipf(n_experts: int = 64, s: float = 1.1, seed: int = 4) -> torch.Tensor:
    """Per-expert router-logit offset of the skewed-load workload: b_e = log(p_e * E) with
    p_e proportional to rank_e^-s over a seeded permutation of the experts."""
    g = torch.Generator().manual_seed(seed)
    ranks = torch.randperm(n_experts, generator=g).float() + 1.0
    p = ranks.pow(-s)
    p = p / p.sum()
    return torch.log(p * n_experts).float()


def add_router_bias(model: DeepseekV2ForCausalLM, bias: torch.Tensor) -> None:
    """Add `bias` to every MoE layer's fp32 router logits before the softmax: HF's MoE
    forward computes the logits inline (modeling_deepseek_v2.py:123-127) and hands them to
    route_tokens_to_experts, which this wraps."""
    for layer in model.model.layers:
        mlp = layer.mlp
        if not hasattr(mlp, "route_tokens_to_experts"):
            continue
        b = bias.to(device=mlp.gate.weight.device, dtype=torch.float32)
        orig = mlp.route_tokens_to_experts

        def route(router_logits, _orig=orig, _b=b):
            return _orig(router_logits + _b)

        mlp.route_tokens_to_experts = route


__all__ = ["YARN", "ARCH", "dsv2_lite_config", "build_model", "router_bias_zipf", "add_router_bias"]
