"""Absorbed-MLA decode attention shared by attention_decode_small and attention_decode_batch.

Reference: AttentionPackedWeights / pack_attention_weights (attention_decode_small.py:24-34,
:426-449; the batch module re-exports the same packing, attention_decode_batch.py:214-237)
and the per-call pipeline of attention_decode_only_triton (:553-674).

The reference materialises per-head K [B,16,S,192] / V [B,16,S,128]; this build keeps
the 576-wide latent row per position ([RMSNorm(c_kv) * w | RoPE(k_pe)]) and absorbs the
kv_b projection into the query and the output:
    q_abs[b,h] = W_UK[h]^T q_nope[b,h]       (W_UK[h] = kv_b[h*256 : h*256+128])
    o_lat[b,h] = softmax(scale * (q_abs . latent + q_pe . k_pe)) @ latent
    o[b, h*128:(h+1)*128] = W_UV[h] o_lat[b,h]  (W_UV[h] = kv_b[h*256+128 : h*256+256])
which equals the expanded computation up to rounding.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

from .. import ops

HIDDEN, HEADS, QK_NOPE, QK_ROPE, V_DIM, KV_LORA = 2048, 16, 128, 64, 128, 512
Q_DIM = QK_NOPE + QK_ROPE
Q_ROWS = HEADS * Q_DIM                  # 3072
KV_A_ROWS = KV_LORA + QK_ROPE           # 576
QKVA_ROWS = Q_ROWS + KV_A_ROWS          # 3648
KVB_ROWS = HEADS * (QK_NOPE + V_DIM)    # 4096
LATENT_ROW = KV_A_ROWS                  # cache row width


@dataclass
class AttentionDecodeWorkspace:
    qkva: torch.Tensor      # [B, 3648] bf16: q (16 x 192) ++ kv_a (512 latent + 64 k_pe)
    q_pe: torch.Tensor      # [B, 16, 64] roped q_pe
    q_nope: torch.Tensor    # [B, 16, 128]
    q_abs: torch.Tensor     # [B, 16, 512]
    o_part: torch.Tensor    # [B, n_splits, 16, 512] fp32 attention partials
    ml_part: torch.Tensor   # [B, n_splits, 16, 2] fp32 (max, sum) per partial
    row_sync: torch.Tensor  # [B] int32 merge tickets (zero between calls)
    o_lat: torch.Tensor     # [B, 16, 512]
    attn_o: torch.Tensor    # [B, 2048] (16 heads x 128)
    o_out: torch.Tensor     # [B, 2048] returned as [B, 1, 2048]
    split_len: int


@dataclass
class AttentionPackedWeights:
    # Q and KV-A packed together: [3648, 2048]
    q_kv_a_weight: torch.Tensor
    # KV-B packed as [4096, 512]
    kv_b_weight: torch.Tensor
    # O: [2048, 2048]
    o_weight: torch.Tensor
    kv_a_ln_weight: torch.Tensor
    kv_a_ln_eps: float
    # absorbed query projection W_UK^T per head [16, 512, 128]
    w_uk_t: torch.Tensor | None = None
    workspace_by_device: dict = field(default_factory=dict)


def pack_attention_weights(attn: torch.nn.Module) -> AttentionPackedWeights:
    """Pack an MLA attention module (checkpoint modeling code or transformers' native
    DeepseekV2Attention; shapes are read from the weights)."""
    q = getattr(attn, "q_proj", None)
    if q is None or getattr(attn, "q_a_proj", None) is not None:
        raise NotImplementedError("attention decode is specialized for DeepSeek-V2-Lite (no q-LoRA)")
    qw = q.weight
    kva = attn.kv_a_proj_with_mqa.weight
    kvb = attn.kv_b_proj.weight
    ow = attn.o_proj.weight
    if (tuple(qw.shape) != (Q_ROWS, HIDDEN) or tuple(kva.shape) != (KV_A_ROWS, HIDDEN)
            or tuple(kvb.shape) != (KVB_ROWS, KV_LORA) or tuple(ow.shape) != (HIDDEN, HEADS * V_DIM)):
        raise NotImplementedError("attention_decode_only_triton is specialized for DeepSeek-V2-Lite dimensions")
    for name in ("q_proj", "kv_a_proj_with_mqa", "o_proj"):
        if getattr(getattr(attn, name), "bias", None) is not None:
            raise NotImplementedError("attention projections with bias are not supported")
    kv_b = kvb.contiguous()
    w_uk_t = kv_b.view(HEADS, QK_NOPE + V_DIM, KV_LORA)[:, :QK_NOPE, :].transpose(1, 2).contiguous()
    ln = attn.kv_a_layernorm
    eps = getattr(ln, "variance_epsilon", getattr(ln, "eps", 1e-6))
    return AttentionPackedWeights(
        q_kv_a_weight=torch.cat((qw, kva), dim=0).contiguous(),
        kv_b_weight=kv_b,
        o_weight=ow.contiguous(),
        kv_a_ln_weight=ln.weight.contiguous(),
        kv_a_ln_eps=float(eps),
        w_uk_t=w_uk_t,
    )


def _workspace(packed: AttentionPackedWeights, dev: torch.device, B: int, max_len: int,
               family: int) -> AttentionDecodeWorkspace:
    key = (dev.index if dev.index is not None else 0, B, max_len, family)
    ws = packed.workspace_by_device.get(key)
    if ws is not None:
        return ws
    from ..engine import choose_split_len
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    split_len = choose_split_len(B, max_len, sms)
    n_splits = ops.mla_splits(B, max_len, split_len, sms)
    bf, f32 = torch.bfloat16, torch.float32
    ws = AttentionDecodeWorkspace(
        qkva=torch.empty((B, QKVA_ROWS), device=dev, dtype=bf),
        q_pe=torch.empty((B, HEADS, QK_ROPE), device=dev, dtype=bf),
        q_nope=torch.empty((B, HEADS, QK_NOPE), device=dev, dtype=bf),
        q_abs=torch.empty((B, HEADS, KV_LORA), device=dev, dtype=bf),
        o_part=torch.empty((B, n_splits, HEADS, KV_LORA), device=dev, dtype=f32),
        ml_part=torch.empty((B, n_splits, HEADS, 2), device=dev, dtype=f32),
        row_sync=torch.zeros(B, device=dev, dtype=torch.int32),
        o_lat=torch.empty((B, HEADS, KV_LORA), device=dev, dtype=bf),
        attn_o=torch.empty((B, HEADS * V_DIM), device=dev, dtype=bf),
        o_out=torch.empty((B, HIDDEN), device=dev, dtype=bf),
        split_len=split_len,
    )
    packed.workspace_by_device[key] = ws
    return ws


def _rope_table(t: torch.Tensor, name: str) -> torch.Tensor:
    if t.ndim != 2 or t.shape[1] < QK_ROPE // 2:
        raise ValueError(f"{name} must be [max_position, >= 32] (the first 32 columns are read)")
    if t.dtype != torch.float32 or t.stride(1) != 1:
        t = t.to(torch.float32).contiguous()
    return t


def mla_decode_layer(name: str, hidden_states, cos, sin, position_ids, cache_position, key_cache,
                     value_cache, packed: AttentionPackedWeights, softmax_scale: float, family: int,
                     single_row: bool) -> torch.Tensor:
    """One q_len=1 attention sublayer for every row of hidden_states [B, 1, 2048]:
    projections, latent-cache write at the row's position, attention over positions
    [0, pos], output projection.  Returns the workspace output [B, 1, 2048] (reused by
    the next call with the same batch size, as the reference's workspace is)."""
    if hidden_states.device.type != "cuda":
        raise NotImplementedError(f"{name} requires CUDA tensors")
    if hidden_states.dtype != torch.bfloat16:
        raise NotImplementedError(f"{name} supports bf16 only")
    if single_row:
        if tuple(hidden_states.shape) != (1, 1, HIDDEN):
            raise ValueError("hidden_states shape must be [1,1,2048]")
    elif hidden_states.ndim != 3 or hidden_states.shape[1] != 1 or hidden_states.shape[2] != HIDDEN:
        raise ValueError("hidden_states shape must be [B,1,2048]")
    B = int(hidden_states.shape[0])
    if position_ids.ndim != 2 or position_ids.shape != (B, 1) or position_ids.dtype != torch.long:
        raise ValueError(f"position_ids must be CUDA int64 tensor with shape [{B},1]")
    if cache_position.numel() not in (1, B) or cache_position.dtype != torch.long:
        raise ValueError("cache_position must be CUDA int64 tensor with one element (or one per row)")
    if (key_cache.ndim != 3 or key_cache.shape[0] != B or key_cache.shape[2] != LATENT_ROW
            or key_cache.dtype != torch.bfloat16):
        raise NotImplementedError(f"{name}: key_cache must be the bf16 latent cache [B, S, 576]")
    if key_cache.stride(2) != 1 or key_cache.stride(1) != LATENT_ROW:
        raise NotImplementedError(f"{name}: key_cache rows must be contiguous")
    if packed.w_uk_t is None:
        raise ValueError("packed attention weights lack the absorbed W_UK (use pack_attention_weights)")
    cos = _rope_table(cos, "cos")
    sin = _rope_table(sin, "sin")
    x = hidden_states.view(B, HIDDEN)
    if x.stride(1) != 1 or x.stride(0) % 8:
        x = x.contiguous()
    dev = x.device
    max_len = int(key_cache.shape[1])
    ws = _workspace(packed, dev, B, max_len, family)
    pos = cache_position.reshape(-1)
    if not pos.is_contiguous():
        pos = pos.contiguous()
    ops.linear(w=packed.q_kv_a_weight, n_rows=QKVA_ROWS, k=HIDDEN, x=x, y=ws.qkva, n_tokens=B,
               family=family, x_group_rows=B)
    ops.mla_prep(qkva=ws.qkva, kv_norm_w=packed.kv_a_ln_weight, eps=packed.kv_a_ln_eps, cos=cos, sin=sin,
                 positions=pos, cache=key_cache, q_pe_out=ws.q_pe, q_nope_out=ws.q_nope)
    ops.linear(w=packed.w_uk_t, n_rows=KV_LORA, k=QK_NOPE, w_row_stride=QK_NOPE,
               w_group_stride=KV_LORA * QK_NOPE, x=ws.q_nope, x_row_stride=HEADS * QK_NOPE,
               x_group_stride=QK_NOPE, y=ws.q_abs, y_row_stride=HEADS * KV_LORA, y_group_stride=KV_LORA,
               n_groups=HEADS, n_tokens=B, family=family, w_group_rows=KV_LORA, x_group_rows=B)
    ops.mla_decode(q_abs=ws.q_abs, q_pe=ws.q_pe, cache=key_cache, positions=pos, softmax_scale=softmax_scale,
                   split_len=ws.split_len, o_part=ws.o_part, ml_part=ws.ml_part, o_lat=ws.o_lat,
                   inputs_prior=True, row_sync=ws.row_sync)
    kv_b = packed.kv_b_weight
    ops.linear(w=kv_b[QK_NOPE:], n_rows=V_DIM, k=KV_LORA, w_row_stride=KV_LORA,
               w_group_stride=(QK_NOPE + V_DIM) * KV_LORA, x=ws.o_lat, x_row_stride=HEADS * KV_LORA,
               x_group_stride=KV_LORA, y=ws.attn_o, y_row_stride=HEADS * V_DIM, y_group_stride=V_DIM,
               n_groups=HEADS, n_tokens=B, family=family, w_group_rows=V_DIM, x_group_rows=B)
    ops.linear(w=packed.o_weight, n_rows=HIDDEN, k=HEADS * V_DIM, x=ws.attn_o, y=ws.o_out, n_tokens=B,
               family=family, x_group_rows=B)
    return ws.o_out.view(B, 1, HIDDEN)
