"""CPU restatement of the decode path's operators (fp32 torch, float64 where noted).

TEST INFRASTRUCTURE ONLY.  Imported by tests/, __graft_entry__.smoke() and the
CPU-baseline / reference arms of bench.py as the checker; the product never calls it.

Every function cites the reference code it restates:
  REF = heiheiha798/Flash-DeepSeeek-V2-Lite (triton_kernels/*, src/run.py)
  HF  = transformers 5.5.0 models/deepseek_v2/modeling_deepseek_v2.py (the oracle model)
Parity is pinned by tests/golden/ fixtures produced by the reference's own Triton
kernels (run by the Triton CPU interpreter) and by the HF model; see
tests/golden/make_golden.py.
"""
from __future__ import annotations

import math

import torch

BF16 = torch.bfloat16


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """REF rmsnorm.py:8-57: y = x * rsqrt(mean(x^2) + eps) * w in fp32, one rounding to x.dtype."""
    xf = x.float()
    inv = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return (xf * inv * w.float()).to(x.dtype)


def residual_add(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """REF attention_prepost.py:85-110: fp32 add, result in the inputs' dtype (bf16 / fp16)."""
    return (a.float() + b.float()).to(a.dtype)


def silu_mul(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """REF mlp_elementwise.py:8-21: silu(g) * u in fp32, bf16 result."""
    g = gate.float()
    return (g * torch.sigmoid(g) * up.float()).to(BF16)


def add_rmsnorm(h: torch.Tensor, delta: torch.Tensor | None, w: torch.Tensor, eps: float):
    """Residual add (REF attention_prepost.py:85-110) followed by RMSNorm (REF rmsnorm.py).
    delta: bf16 [R, C] or fp32 per-slot partials [R, P, C] summed in fp32 first."""
    if delta is None:
        hn = h
    elif delta.dim() == 3:
        hn = (h.float() + delta.float().sum(1)).to(BF16)
    else:
        hn = residual_add(h, delta)
    return hn, rmsnorm(hn, w, eps)


def prepare_decode_inputs(cache_position: torch.Tensor, mask_index: torch.Tensor, batch: int):
    """REF attention_prepost.py:8-36: mask[b, s] = (index[s] <= pos_b), position_ids[b] = pos_b."""
    pos = cache_position.view(-1)
    if pos.numel() == 1:
        pos = pos.expand(batch)
    mask = (mask_index.view(1, -1) <= pos.view(-1, 1)).long()
    return mask, pos.view(-1, 1).clone()


def copy_single_token_to_cache(src: torch.Tensor, dst: torch.Tensor, cache_position: torch.Tensor):
    """REF attention_prepost.py:39-82: dst[b, h, pos_b, :] = src[b, h, 0, :] (in place)."""
    pos = cache_position.view(-1)
    for b in range(src.shape[0]):
        p = int(pos[0 if pos.numel() == 1 else b])
        dst[b, :, p, :] = src[b, :, 0, :]
    return dst


def softmax_topk6(logits: torch.Tensor, scaling: float):
    """REF moe_router.py:8-60: softmax over the experts, six rounds of (max, argmax, mask),
    lowest index first on ties; weights multiplied by routed_scaling_factor."""
    p = torch.softmax(logits.float(), dim=-1)
    ids = torch.empty(p.shape[0], 6, dtype=torch.long)
    w = torch.empty(p.shape[0], 6, dtype=torch.float32)
    for r in range(p.shape[0]):
        work = p[r].clone()
        for k in range(6):
            m = work.max()
            i = int(torch.nonzero(work == m)[0])
            ids[r, k] = i
            w[r, k] = m * scaling
            work[i] = -math.inf
    return ids, w


def router(x: torch.Tensor, gate_w: torch.Tensor, scaling: float, bias: torch.Tensor | None = None):
    """HF :123-127 + :100-120 (greedy): logits = fp32(x) @ fp32(W)^T (+ bias), softmax, top-6."""
    logits = x.float() @ gate_w.float().t()
    if bias is not None:
        logits = logits + bias.float()
    ids, w = softmax_topk6(logits, scaling)
    return logits, ids, w


def bucket(ids: torch.Tensor, weights: torch.Tensor, expert_lo: int, n_local: int, shared_lo: int,
           shared_hi: int):
    """Stable counting sort of routes r = b*6 + k by local expert (REF moe_batch.py:101-148
    buckets with atomics; the restated order is ascending (token, k)), followed by two
    shared-expert groups of rows [shared_lo, shared_hi) with weight 1 and slots b*8+6, b*8+7."""
    rows = ids.shape[0]
    groups = [[] for _ in range(n_local)]
    for r in range(rows * 6):
        e = int(ids.view(-1)[r]) - expert_lo
        if 0 <= e < n_local:
            b, k = divmod(r, 6)
            groups[e].append((b, b * 8 + k, float(weights.view(-1)[r])))
    for s in range(2):
        groups.append([(b, b * 8 + 6 + s, 1.0) for b in range(shared_lo, shared_hi)])
    offsets = [0]
    for g in groups:
        offsets.append(offsets[-1] + len(g))
    flat = [t for g in groups for t in g]
    tok = torch.tensor([t[0] for t in flat], dtype=torch.int32)
    slot = torch.tensor([t[1] for t in flat], dtype=torch.int32)
    wt = torch.tensor([t[2] for t in flat], dtype=torch.float32)
    return torch.tensor(offsets, dtype=torch.int32), tok, slot, wt


def expert_mlp(x: torch.Tensor, gate_up: torch.Tensor, down: torch.Tensor) -> torch.Tensor:
    """HF :61-79 per-expert MLP in bf16 semantics: gate/up linear outputs rounded to bf16,
    silu(gate) * up rounded to bf16, down linear output rounded to bf16 (fp32 accumulation)."""
    inter = gate_up.shape[0] // 2
    gu = (x.float() @ gate_up.float().t()).to(BF16)
    g, u = gu[:, :inter], gu[:, inter:]
    h = (torch.nn.functional.silu(g.float()).to(BF16).float() * u.float()).to(BF16)
    return (h.float() @ down.float().t()).to(BF16)


def moe(x: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor, gate_up: torch.Tensor,
        down: torch.Tensor, shared_gate: torch.Tensor, shared_up: torch.Tensor,
        shared_down: torch.Tensor) -> torch.Tensor:
    """HF DeepseekV2Moe.forward (:121-128) + DeepseekV2Experts.forward (:58-80) in fp32 sums:
    out = sum_k w_k * expert_{id_k}(x) + shared_mlp(x)  (returned in fp32).  Like HF's eager
    experts loop, each expert hit runs once over all of its routed rows, and its weighted
    outputs are added to their rows in fp32.  Runs on the tensors' device."""
    out = torch.zeros(x.shape[0], x.shape[1], dtype=torch.float32, device=x.device)
    ids = ids.to(x.device)
    weights = weights.to(x.device)
    flat = ids.reshape(-1)
    for e in torch.unique(flat).tolist():
        r = torch.nonzero(flat == e).flatten()
        b = r // ids.shape[1]
        y = expert_mlp(x[b], gate_up[e], down[e]).float()
        out.index_add_(0, b, y * weights.reshape(-1)[r].float().view(-1, 1))
    sh = expert_mlp(x, torch.cat([shared_gate, shared_up], 0), shared_down)
    return out + sh.float()


def rope_interleaved(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """HF apply_rotary_emb (:271-284): rotate pairs (2j, 2j+1) by angle j, fp32 math,
    output in the input dtype.  cos/sin [.., 32] already include attention_scaling."""
    xf = x.float()
    e, o = xf[..., 0::2], xf[..., 1::2]
    re = e * cos - o * sin
    im = o * cos + e * sin
    return torch.stack([re, im], -1).flatten(-2).to(x.dtype)


def rope_half_split(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """REF _build_qkv_rope_kernel (attention_decode_small.py:190-229): same rotation as
    rope_interleaved, output in DeepSeek half-split order [rotated evens | rotated odds]."""
    r = rope_interleaved(x, cos, sin).float()
    return torch.cat([r[..., 0::2], r[..., 1::2]], -1).to(x.dtype)


def latent_row(kva: torch.Tensor, norm_w: torch.Tensor, eps: float, cos: torch.Tensor,
               sin: torch.Tensor) -> torch.Tensor:
    """Latent cache row from kv_a_proj_with_mqa output [.., 576]:
    [rmsnorm(c_kv) * w (REF rmsnorm formula) | rope(k_pe)]  (bf16)."""
    lat = rmsnorm(kva[..., :512].to(BF16), norm_w, eps)
    return torch.cat([lat, rope_interleaved(kva[..., 512:].to(BF16), cos, sin)], -1)


def mla_decode(q_abs: torch.Tensor, q_pe: torch.Tensor, cache: torch.Tensor, lengths, scale: float):
    """Absorbed-MLA q_len=1 attention over the latent cache (float64 reference):
    score[h, s] = scale * (q_abs[h] . cache[s, :512] + q_pe[h] . cache[s, 512:]), s < len_b;
    o_lat[h] = softmax(score[h]) @ cache[:len, :512].  q_abs/q_pe [B, 16, 512/64],
    cache [B, S, 576].  Equals REF _batched_decode_attention_q1_kernel
    (attention_decode_batch.py:240-342) on the expanded K = [W_UK c | k_pe], V = W_UV c."""
    B = q_abs.shape[0]
    out = torch.zeros(B, q_abs.shape[1], 512, dtype=torch.float64)
    for b in range(B):
        n = int(lengths[b])
        kv = cache[b, :n].double()
        q = torch.cat([q_abs[b].double(), q_pe[b].double()], -1)
        s = (q @ kv.t()) * scale
        p = torch.softmax(s, dim=-1)
        out[b] = p @ kv[:, :512]
    return out


def expanded_attention_decode(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, lengths, scale: float):
    """REF _batched_decode_attention_q1_kernel (attention_decode_batch.py:240-342):
    q [B, H, 192], K [B, H, S, 192], V [B, H, S, 128]; attends positions < len_b."""
    B, H = q.shape[:2]
    out = torch.zeros(B, H, v.shape[-1], dtype=torch.float64)
    for b in range(B):
        n = int(lengths[b])
        s = torch.einsum("hd,hsd->hs", q[b].double(), k[b, :, :n].double()) * scale
        p = torch.softmax(s, -1)
        out[b] = torch.einsum("hs,hsd->hd", p, v[b, :, :n].double())
    return out


def absorbed_attention_layer(x: torch.Tensor, attn, cache: torch.Tensor, pos: torch.Tensor,
                             cos_tab: torch.Tensor, sin_tab: torch.Tensor, scale: float):
    """One decode step of an HF DeepseekV2Attention (HF :337-395) in the absorbed latent
    form used by the engine.  x [B, 2048] (normed input), cache [B, S, 576] is updated in
    place at pos[b]; returns the o_proj output [B, 2048] (bf16-rounded stages like the engine)."""
    B = x.shape[0]
    qkva = (x.float() @ torch.cat([attn.q_proj.weight, attn.kv_a_proj_with_mqa.weight], 0).float().t()).to(BF16)
    q = qkva[:, :3072].view(B, 16, 192)
    kva = qkva[:, 3072:]
    kv_b = attn.kv_b_proj.weight.float().view(16, 256, 512)
    q_abs = torch.einsum("bhd,hdc->bhc", q[..., :128].float(), kv_b[:, :128]).to(BF16)
    q_pe = torch.empty(B, 16, 64, dtype=BF16)
    for b in range(B):
        p = int(pos[b])
        cache[b, p] = latent_row(kva[b], attn.kv_a_layernorm.weight, attn.kv_a_layernorm.variance_epsilon,
                                 cos_tab[p], sin_tab[p])
        q_pe[b] = rope_interleaved(q[b, :, 128:], cos_tab[p], sin_tab[p])
    o_lat = mla_decode(q_abs, q_pe, cache, pos + 1, scale).to(BF16)
    o = torch.einsum("bhc,hvc->bhv", o_lat.float(), kv_b[:, 128:]).to(BF16).reshape(B, 2048)
    return (o.float() @ attn.o_proj.weight.float().t()).to(BF16)


def linear(w: torch.Tensor, x: torch.Tensor, epilogue: str = "bf16", up: torch.Tensor | None = None,
           scale: torch.Tensor | None = None) -> torch.Tensor:
    """y = x @ w^T with the engine's epilogues: 'bf16', 'f32', 'swiglu' (bf16(silu(bf16 g) * bf16 u)),
    'scale' (bf16(acc) * scale[row], fp32).  Restates REF _batched_linear_kernel
    (attention_decode_batch.py:420-468) and the grouped MoE epilogues (moe_batch.py:151-307)."""
    acc = x.float() @ w.float().t()
    if epilogue == "bf16":
        return acc.to(BF16)
    if epilogue == "f32":
        return acc
    if epilogue == "swiglu":
        u = (x.float() @ up.float().t()).to(BF16).float()
        g = acc.to(BF16).float()
        return (g * torch.sigmoid(g) * u).to(BF16)
    if epilogue == "scale":
        return acc.to(BF16).float() * scale.view(-1, 1).float()
    raise ValueError(epilogue)
