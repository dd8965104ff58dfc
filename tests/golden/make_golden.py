"""Generate the golden fixtures that pin the oracle (oracle/ops.py) to the reference.

Run where the reference checkout is available (its directory in DSV2_REFERENCE) with the
Triton CPU interpreter:

    DSV2_REFERENCE=<reference checkout> TRITON_INTERPRET=1 python tests/golden/make_golden.py

Outputs (committed):
  tests/golden/ref_kernels.pt  inputs and outputs of the reference's own Triton kernels
                               (heiheiha798/Flash-DeepSeeek-V2-Lite, triton_kernels/*),
                               launched with the reference wrappers' grid/tile parameters
                               on CPU tensors through the Triton interpreter.
  tests/golden/hf_config1.pt   BASELINE config 1 run through the HF eager DeepSeek-V2
                               (transformers 5.5.0): 2 layers, fp32, seed 0, 128-token
                               prompt, 16 greedy q_len=1 decode steps: generated ids,
                               per-layer hidden states and router ids of the first decode
                               step, and its logits.
The reference's batch-family grouped MoE kernels dot raw bf16 tiles, which the Triton
3.6 interpreter mis-evaluates, and its small-family MoE computes a mis-indexed SwiGLU;
MoE parity is therefore pinned to the HF model (hf_config1.pt) instead.
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
REF = Path(os.environ.get("DSV2_REFERENCE", str(REPO.parent / "reference")))


def ref_kernels() -> dict:
    assert os.environ.get("TRITON_INTERPRET") == "1", "run with TRITON_INTERPRET=1"
    sys.path.insert(0, str(REF))
    from triton_kernels import attention_decode_batch as AB
    from triton_kernels import attention_decode_small as AS
    from triton_kernels import attention_prepost as P
    from triton_kernels import mlp_elementwise as M
    from triton_kernels import moe_router as R
    from triton_kernels import rmsnorm as N

    g = torch.Generator().manual_seed(1234)
    out: dict = {}

    # rmsnorm.py:60-95 launch: grid (rows,), BLOCK_COL 512, num_warps 4
    for name, rows, cols in (("rmsnorm_2048", 5, 2048), ("rmsnorm_512", 3, 512)):
        x = (torch.randn(rows, cols, generator=g) * 3).to(torch.bfloat16)
        w = (1 + 0.1 * torch.randn(cols, generator=g)).to(torch.bfloat16)
        y = torch.empty_like(x)
        N._rmsnorm_kernel[(rows,)](x, w, y, cols, 1e-6, x.stride(0), x.stride(1), y.stride(0), y.stride(1),
                                   BLOCK_COL=512, num_warps=4)
        out[name] = dict(x=x, w=w, eps=1e-6, y=y)

    # attention_prepost.py:191-223: grid (rows, cdiv(cols, 256))
    a = torch.randn(4, 2048, generator=g).to(torch.bfloat16)
    b = torch.randn(4, 2048, generator=g).to(torch.bfloat16)
    o = torch.empty_like(a)
    P._residual_add_kernel[(4, 8)](a, b, o, 2048, a.stride(0), a.stride(1), b.stride(0), b.stride(1),
                                   o.stride(0), o.stride(1), BLOCK_COL=256, num_warps=4)
    out["residual_add"] = dict(a=a, b=b, out=o)

    # mlp_elementwise.py:24-45: grid cdiv(n, 1024)
    gt = (torch.randn(3, 1408, generator=g) * 2).to(torch.bfloat16)
    up = torch.randn(3, 1408, generator=g).to(torch.bfloat16)
    o = torch.empty_like(gt)
    M._silu_mul_kernel[((gt.numel() + 1023) // 1024,)](gt, up, o, gt.numel(), BLOCK=1024, num_warps=4)
    out["silu_mul"] = dict(gate=gt, up=up, out=o)

    # moe_router.py:63-86 on [1, 64] logits, one launch per row; row 0 carries an exact tie
    logits = torch.randn(8, 64, generator=g)
    logits[0, 10] = logits[0, 20] = logits[0].max() + 0.5
    ids = torch.empty(8, 6, dtype=torch.long)
    wts = torch.empty(8, 6)
    for r in range(8):
        i1 = torch.empty(1, 6, dtype=torch.long)
        w1 = torch.empty(1, 6)
        R._router_softmax_topk6_kernel[(1,)](logits[r:r + 1].contiguous(), i1, w1, scaling=1.0, BLOCK_E=64,
                                            num_warps=2)
        ids[r], wts[r] = i1[0], w1[0]
    out["router_topk6"] = dict(logits=logits, scaling=1.0, ids=ids, weights=wts)

    # attention_prepost.py:152-188: grid (B, cdiv(max_len, 256))
    B, S = 3, 300
    pos = torch.tensor([137], dtype=torch.long)
    mask = torch.empty(B, S, dtype=torch.long)
    pid = torch.empty(B, 1, dtype=torch.long)
    idx = torch.arange(S, dtype=torch.long)
    P._prepare_decode_inputs_kernel[(B, 2)](pos, mask, pid, idx, S, B, mask.stride(0), mask.stride(1),
                                            pid.stride(0), pid.stride(1), BLOCK=256, num_warps=2)
    out["prepare_decode_inputs"] = dict(cache_position=pos, attention_mask_index=idx, batch=B,
                                        attention_mask=mask, position_ids=pid)

    # attention_prepost.py:113-149: grid (B, H, cdiv(D, 128))
    src = torch.randn(2, 16, 1, 192, generator=g).to(torch.bfloat16)
    dst0 = torch.randn(2, 16, 40, 192, generator=g).to(torch.bfloat16)
    dst = dst0.clone()
    cp = torch.tensor([17], dtype=torch.long)
    P._cache_write_q1_kernel[(2, 16, 2)](src, dst, cp, 16, 192, *src.stride(), *dst.stride(), BLOCK_D=128,
                                         num_warps=2)
    out["copy_single_token_to_cache"] = dict(src=src, dst_before=dst0, cache_position=cp, dst_after=dst)

    # attention_decode_small.py:585-616 RoPE (half-split output) via _build_qkv_rope_kernel, B = 1
    H = 16
    q_proj = torch.randn(H, 192, generator=g).to(torch.bfloat16)
    kvb = torch.randn(H, 256, generator=g).to(torch.bfloat16)
    k_pe = torch.randn(64, generator=g).to(torch.bfloat16)
    max_len = 64
    inv = 1.0 / (10000 ** (torch.arange(0, 64, 2).float() / 64))
    fr = torch.arange(max_len).float()[:, None] * inv[None, :]
    cos = torch.cat([fr.cos(), fr.cos()], -1)
    sin = torch.cat([fr.sin(), fr.sin()], -1)
    pid1 = torch.tensor([23], dtype=torch.long)
    q_out = torch.empty(H, 192, dtype=torch.bfloat16)
    k_new = torch.empty(H, 192, dtype=torch.bfloat16)
    v_new = torch.empty(H, 128, dtype=torch.bfloat16)
    AS._build_qkv_rope_kernel[(H, 3)](q_proj, kvb, k_pe, cos, sin, pid1, q_out, k_new, v_new, H, 192, 128, 64,
                                      128, q_proj.stride(0), q_proj.stride(1), kvb.stride(0), kvb.stride(1),
                                      cos.stride(0), cos.stride(1), sin.stride(0), sin.stride(1),
                                      q_out.stride(0), q_out.stride(1), k_new.stride(0), k_new.stride(1),
                                      v_new.stride(0), v_new.stride(1), BLOCK_D=64, num_warps=4)
    out["build_qkv_rope"] = dict(q_proj=q_proj, kvb_proj=kvb, k_pe=k_pe, cos=cos, sin=sin, position=pid1,
                                 q_out=q_out, k_new=k_new, v_new=v_new)

    # attention_decode_batch.py:345-400: grid (B, H, cdiv(128, 128)), BLOCK_N 32
    B, H, S = 2, 16, 80
    q = (torch.randn(B, H, 1, 192, generator=g) * 0.5).to(torch.bfloat16)
    k = (torch.randn(B, H, S, 192, generator=g) * 0.5).to(torch.bfloat16)
    v = torch.randn(B, H, S, 128, generator=g).to(torch.bfloat16)
    cp = torch.tensor([70], dtype=torch.long)
    o = torch.empty(B, H, 1, 128, dtype=torch.bfloat16)
    scale = 192 ** -0.5
    AB._batched_decode_attention_q1_kernel[(B, H, 1)](q, k, v, cp, o, 192, 128, *q.stride(), *k.stride(),
                                                      *v.stride(), *o.stride(), scale, BLOCK_N=32, BLOCK_Q=64,
                                                      BLOCK_V=128, num_warps=4)
    out["batched_attention"] = dict(q=q, k=k, v=v, cache_position=cp, scale=scale, out=o)
    return out


@torch.no_grad()
def hf_config1() -> dict:
    sys.path.insert(0, str(REPO))
    from transformers import DynamicCache

    from oracle.hf_model import build_model, dsv2_lite_config

    torch.manual_seed(0)
    cfg = dsv2_lite_config(num_layers=2)
    model = build_model(cfg, seed=0, device="cpu", dtype=torch.float32)
    prompt = torch.randint(0, cfg.vocab_size, (1, 128), generator=torch.Generator().manual_seed(0))
    routes: list[torch.Tensor] = []
    moe = model.model.layers[1].mlp
    orig = moe.route_tokens_to_experts

    def record(logits):
        ids, w = orig(logits)
        routes.append(ids.clone())
        return ids, w

    moe.route_tokens_to_experts = record
    cache = DynamicCache(config=cfg)
    out = model(input_ids=prompt, past_key_values=cache, use_cache=True)
    tok = out.logits[:, -1].argmax(-1, keepdim=True)
    generated = [int(tok)]
    routes.clear()
    hidden = logits1 = None
    step_routes = []
    for step in range(16):
        out = model(input_ids=tok, past_key_values=cache, use_cache=True, output_hidden_states=(step == 0))
        if step == 0:
            hidden = torch.stack([h[0, -1] for h in out.hidden_states])
            logits1 = out.logits[0, -1].clone()
        step_routes.append(routes[-1].view(-1).clone())
        tok = out.logits[:, -1].argmax(-1, keepdim=True)
        generated.append(int(tok))
    return dict(seed=0, num_layers=2, prompt=prompt[0], generated=torch.tensor(generated),
                hidden_step1=hidden, logits_step1=logits1, routes=torch.stack(step_routes))


if __name__ == "__main__":
    torch.save(ref_kernels(), HERE / "ref_kernels.pt")
    torch.save(hf_config1(), HERE / "hf_config1.pt")
    for f in ("ref_kernels.pt", "hf_config1.pt"):
        print(f, (HERE / f).stat().st_size)
