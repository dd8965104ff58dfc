"""Synthetic DeepSeek-V2-Lite model: the transformers (5.5) DeepseekV2ForCausalLM with the
benchmark's shapes and seeded random weights.

The reference runner loads DeepSeek-V2-Lite-Chat with the checkpoint's remote modeling
code (src/run.py:719-725).  No checkpoint or network is available to this build, so
benchmarks, the runner CLI and the tests use this stand-in: the same architecture as the
reference's hard-coded constants (triton_kernels/attention_decode_small.py:12-21) with
hidden 2048, 16 heads, MLA without q-LoRA, kv_lora_rank 512, qk_nope 128, qk_rope 64,
v_head 128, 64 routed experts of intermediate 1408, top-6 greedy softmax routing, 2
shared experts, layer 0 dense (intermediate 10944), vocab 102400, RMSNorm eps 1e-6,
YaRN RoPE (theta 10000, factor 40).

Weights: N(0, std) for every matrix/embedding, ones for RMSNorm weights, drawn from one
torch.Generator seeded with `seed`, in parameter-registration order, on the target
device, so the same call produces identical weights wherever it runs.  The HF module
is the weight container and runs the eager prefill; the decode step runs in libdsv2.
"""
from __future__ import annotations

import torch
from transformers import DeepseekV2Config, DeepseekV2ForCausalLM
from transformers.initialization import no_init_weights

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


def dsv2_lite_config(num_layers: int = 27, **overrides) -> DeepseekV2Config:
    kw = dict(
        vocab_size=102400,
        hidden_size=2048,
        intermediate_size=10944,
        moe_intermediate_size=1408,
        num_hidden_layers=num_layers,
        num_attention_heads=16,
        num_key_value_heads=16,
        n_shared_experts=2,
        n_routed_experts=64,
        num_experts_per_tok=6,
        routed_scaling_factor=1.0,
        topk_method="greedy",
        norm_topk_prob=False,
        q_lora_rank=None,
        kv_lora_rank=512,
        qk_nope_head_dim=128,
        qk_rope_head_dim=64,
        v_head_dim=128,
        first_k_dense_replace=1,
        max_position_embeddings=163840,
        rms_norm_eps=1e-6,
        rope_parameters=dict(YARN),
        initializer_range=0.02,
        tie_word_embeddings=False,
        bos_token_id=100000,
        eos_token_id=100001,
        pad_token_id=None,
    )
    kw.update(overrides)
    cfg = DeepseekV2Config(**kw)
    cfg._attn_implementation = "eager"
    cfg._experts_implementation = "eager"
    return cfg


@torch.no_grad()
def build_model(cfg: DeepseekV2Config, seed: int, device="cpu", dtype=torch.float32,
                std: float | None = None) -> DeepseekV2ForCausalLM:
    """Instantiate the HF model without HF's own init and fill it deterministically."""
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
    """Per-expert logit offset b_e that skews expert load with Zipf(s) popularity
    (benchmark config 5): b_e = log(p_e / mean p), p_e ~ rank^-s over a seeded
    permutation of the experts."""
    g = torch.Generator().manual_seed(seed)
    ranks = torch.randperm(n_experts, generator=g).float() + 1.0
    p = ranks.pow(-s)
    p = p / p.sum()
    return torch.log(p * n_experts).float()


def add_router_bias(model: DeepseekV2ForCausalLM, bias: torch.Tensor) -> None:
    """Add `bias` to every MoE layer's fp32 router logits before the softmax (the HF MoE
    forward computes the logits inline, modeling_deepseek_v2.py:123-127, so the wrapper
    sits on route_tokens_to_experts).  The engine passes the same tensor to its router."""
    for layer in model.model.layers:
        mlp = layer.mlp
        if not hasattr(mlp, "route_tokens_to_experts"):
            continue
        b = bias.to(device=mlp.gate.weight.device, dtype=torch.float32)
        orig = mlp.route_tokens_to_experts

        def route(router_logits, _orig=orig, _b=b):
            return _orig(router_logits + _b)

        mlp.route_tokens_to_experts = route
