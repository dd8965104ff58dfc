"""DeepSeek-V2-Lite shapes and load-time weight packing for the decode engine.

Packing follows the reference's load-time packers and adds the absorbed-MLA views:
  * attention (attention_decode_small.py:426-449, AttentionPackedWeights :24-34):
    q_proj ++ kv_a_proj_with_mqa -> qkva [3648, 2048]; kv_b [4096, 512]; o [2048, 2048];
    plus W_UK^T per head [16, 512, 128] (w_uk_t[h, c, d] = kv_b[h*256 + d, c]) used to
    absorb q_nope into the 512-wide latent space; W_UV[h] is the strided view
    kv_b[h*256 + 128 : h*256 + 256, :].
  * routed experts (moe_batch.py:324-363, PackedRoutedExperts :12-30): gate_up
    [E, 2*1408, 2048] (gate rows then up rows) and down [E, 2048, 1408]; the two
    shared experts (one MLP of intermediate 2*1408) are appended as two more
    "experts" holding the first / second half of the shared intermediate dimension,
    so sum of both halves == the shared MLP and one grouped launch covers all.
  * dense layer-0 MLP (src/run.py:340-361): gate ++ up -> [2*10944, 2048], down [2048, 10944].
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

HIDDEN = 2048
N_HEADS = 16
QK_NOPE = 128
QK_ROPE = 64
V_DIM = 128
KV_LORA = 512
Q_DIM = QK_NOPE + QK_ROPE            # 192
Q_ROWS = N_HEADS * Q_DIM             # 3072
KV_A_ROWS = KV_LORA + QK_ROPE        # 576
QKVA_ROWS = Q_ROWS + KV_A_ROWS       # 3648
KVB_ROWS = N_HEADS * (QK_NOPE + V_DIM)  # 4096
LATENT_ROW = KV_LORA + QK_ROPE       # 576 (cache row)
TOPK = 6
SLOTS = 8                            # per token: 6 routed + 2 shared-expert halves


def check_config(cfg) -> None:
    """Raise NotImplementedError unless cfg has the DeepSeek-V2-Lite shapes the kernels use."""
    want = dict(hidden_size=HIDDEN, num_attention_heads=N_HEADS, qk_nope_head_dim=QK_NOPE,
                qk_rope_head_dim=QK_ROPE, v_head_dim=V_DIM, kv_lora_rank=KV_LORA)
    bad = {k: getattr(cfg, k, None) for k, v in want.items() if getattr(cfg, k, None) != v}
    if bad:
        raise NotImplementedError(f"decode kernels are specialised for DeepSeek-V2-Lite shapes; got {bad}")
    if getattr(cfg, "q_lora_rank", None) is not None:
        raise NotImplementedError("q-LoRA attention is not part of DeepSeek-V2-Lite")
    if getattr(cfg, "num_experts_per_tok", TOPK) != TOPK:
        raise NotImplementedError("top-6 routing only")
    if getattr(cfg, "topk_method", "greedy") != "greedy" or getattr(cfg, "norm_topk_prob", False):
        raise NotImplementedError("greedy softmax top-k without renormalisation only")


@dataclass
class AttnPack:
    qkva: torch.Tensor        # [3648, 2048]
    kv_norm_w: torch.Tensor   # [512]
    kv_norm_eps: float
    w_uk_t: torch.Tensor      # [16, 512, 128]
    kv_b: torch.Tensor        # [4096, 512]
    o: torch.Tensor           # [2048, 2048]


@dataclass
class DensePack:
    gate_up: torch.Tensor     # [2*I, 2048]
    down: torch.Tensor        # [2048, I]
    inter: int


@dataclass
class MoePack:
    gate_w: torch.Tensor      # [64, 2048]
    gate_bias: torch.Tensor | None  # [64] fp32 logit offset (None = plain HF gate)
    gate_up: torch.Tensor     # [n_local + 2, 2*1408, 2048]
    down: torch.Tensor        # [n_local + 2, 2048, 1408]
    inter: int
    n_experts: int
    expert_lo: int
    n_local: int
    scaling: float


@dataclass
class LayerPack:
    in_norm_w: torch.Tensor
    post_norm_w: torch.Tensor
    eps: float
    attn: AttnPack
    dense: DensePack | None
    moe: MoePack | None


def pack_attention(attn) -> AttnPack:
    q = attn.q_proj.weight
    kva = attn.kv_a_proj_with_mqa.weight
    kv_b = attn.kv_b_proj.weight.contiguous()
    qkva = torch.cat([q, kva], dim=0).contiguous()
    w_uk = kv_b.view(N_HEADS, QK_NOPE + V_DIM, KV_LORA)[:, :QK_NOPE, :]    # [h, d, c]
    w_uk_t = w_uk.transpose(1, 2).contiguous()                            # [h, c, d]
    return AttnPack(qkva=qkva, kv_norm_w=attn.kv_a_layernorm.weight.contiguous(),
                    kv_norm_eps=float(attn.kv_a_layernorm.variance_epsilon), w_uk_t=w_uk_t, kv_b=kv_b,
                    o=attn.o_proj.weight.contiguous())


def pack_dense(mlp) -> DensePack:
    gate_up = torch.cat([mlp.gate_proj.weight, mlp.up_proj.weight], dim=0).contiguous()
    return DensePack(gate_up=gate_up, down=mlp.down_proj.weight.contiguous(),
                     inter=int(mlp.gate_proj.weight.shape[0]))


def pack_moe(moe, expert_lo: int = 0, n_local: int | None = None, alias_hf: bool = False,
             gate_bias: torch.Tensor | None = None) -> MoePack:
    """Pack local routed experts [expert_lo, expert_lo + n_local) plus the shared MLP.

    alias_hf=True (all experts local) rebinds the HF module's expert parameters to
    views of the packed tensor so the weights are stored once.
    """
    ex = moe.experts
    n_exp = int(ex.gate_up_proj.shape[0])
    inter = int(ex.gate_up_proj.shape[1]) // 2
    if n_local is None:
        n_local = n_exp - expert_lo
    sh = moe.shared_experts
    sh_inter = int(sh.gate_proj.weight.shape[0])
    if sh_inter % inter:
        raise NotImplementedError("shared-expert intermediate must be a multiple of the routed one")
    n_sh = sh_inter // inter
    if n_sh != 2:
        raise NotImplementedError("two shared-expert halves expected (n_shared_experts=2)")
    dev, dt = ex.gate_up_proj.device, ex.gate_up_proj.dtype
    G = n_local + n_sh
    gate_up = torch.empty((G, 2 * inter, HIDDEN), device=dev, dtype=dt)
    down = torch.empty((G, HIDDEN, inter), device=dev, dtype=dt)
    gate_up[:n_local].copy_(ex.gate_up_proj.data[expert_lo:expert_lo + n_local])
    down[:n_local].copy_(ex.down_proj.data[expert_lo:expert_lo + n_local])
    for s in range(n_sh):
        rows = slice(s * inter, (s + 1) * inter)
        gate_up[n_local + s, :inter].copy_(sh.gate_proj.weight.data[rows])
        gate_up[n_local + s, inter:].copy_(sh.up_proj.weight.data[rows])
        down[n_local + s].copy_(sh.down_proj.weight.data[:, rows])
    if alias_hf and expert_lo == 0 and n_local == n_exp:
        ex.gate_up_proj.data = gate_up[:n_exp]
        ex.down_proj.data = down[:n_exp]
    return MoePack(gate_w=moe.gate.weight.data, gate_bias=gate_bias, gate_up=gate_up, down=down,
                   inter=inter, n_experts=n_exp, expert_lo=expert_lo, n_local=n_local,
                   scaling=float(moe.routed_scaling_factor))


def pack_layer(layer, expert_lo: int = 0, n_local: int | None = None, alias_hf: bool = False,
               gate_bias: torch.Tensor | None = None) -> LayerPack:
    mlp = layer.mlp
    is_moe = hasattr(mlp, "experts")
    return LayerPack(
        in_norm_w=layer.input_layernorm.weight.data,
        post_norm_w=layer.post_attention_layernorm.weight.data,
        eps=float(layer.input_layernorm.variance_epsilon),
        attn=pack_attention(layer.self_attn),
        dense=None if is_moe else pack_dense(mlp),
        moe=pack_moe(mlp, expert_lo, n_local, alias_hf, gate_bias) if is_moe else None,
    )


def rope_tables(model, max_len: int, device) -> tuple[torch.Tensor, torch.Tensor]:
    """cos/sin [max_len, 32] fp32 from the HF rotary embedding (inv_freq, attention_scaling),
    computed with the same fp32 products as DeepseekV2RotaryEmbedding.forward."""
    rot = model.model.rotary_emb
    inv = rot.inv_freq.to(device=device, dtype=torch.float32)
    pos = torch.arange(max_len, device=device, dtype=torch.float32)
    freqs = pos[:, None] * inv[None, :]
    scale = float(rot.attention_scaling)
    return (torch.cos(freqs) * scale).contiguous(), (torch.sin(freqs) * scale).contiguous()
