"""Same-box timing of the reference's Triton kernels beside this library's kernels (B200).

    python tests/bench_ref_triton.py [--batch 256] [--iters 20]

MEASUREMENT INFRASTRUCTURE, not a test and not the product.  It imports the reference's
unmodified `triton_kernels` package from baseline/_ref/ (the reference is not an
installable package: its files are placed there as they are, outside version control)
and JIT-compiles its kernels for this GPU with the installed Triton.  Each case builds the
same inputs for both sides, replays N launches of each from a CUDA graph (device time,
not host launch rate) and prints one JSON line: time per launch, algorithmic bytes / s and
the ratio, plus the max relative difference between the two outputs where they compute
the same thing.

Cases (shapes of the B=256 decode step):
  moe        reference packed_routed_moe (moe_batch.py:390-557: bucketing, grouped gate_up +
             SwiGLU, grouped down, top-6 reduce; 64 routed experts) vs moe_tc_kernel over the
             same 64 routed experts (bucketing + expert-ordered copy + the fused launch);
  qkva, o    reference _batched_linear_kernel (attention_decode_batch.py:420-468, bf16 out,
             its own tile choice for B >= 128) vs linear_splitk_kernel as the decode step runs
             it (fp32 split-K partials, weights requested before the launch wait) and
             linear_tc_kernel with a bf16 output;
  attention  reference batched_attention_decode_q1_triton (attention_decode_batch.py:240-400)
             over the expanded K [B,16,S,192] / V [B,16,S,128] cache at one shared length
             (its only mode) vs mla_decode_kernel over the 576-wide latent cache, same
             length; and mla_decode at the ragged lengths of the B=256 workload.
"""
from __future__ import annotations

import argparse
import json
import math
import sys
from pathlib import Path

import torch

REPO = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(REPO / "flash-deepseek-v2-lite_b200"))
sys.path.insert(0, str(REPO))
REF = REPO / "baseline" / "_ref"


def graph_time(fn, iters: int, warmup: int = 3) -> float:
    """us per call of fn, replayed `iters` times from one CUDA graph."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(iters):
            fn()
    g.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    g.replay()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) * 1000.0 / iters


def relerr(a, b) -> float:
    a, b = a.double(), b.double()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))


def line(case, ref_us, our_us, nbytes, extra=None):
    d = {"case": case, "ref_us": round(ref_us, 2), "ours_us": round(our_us, 2),
         "ref_GBps": round(nbytes / ref_us / 1e3, 1), "ours_GBps": round(nbytes / our_us / 1e3, 1),
         "speedup": round(ref_us / our_us, 2), "bytes": nbytes}
    d.update(extra or {})
    print(json.dumps(d), flush=True)


def case_moe(B, iters, dev, g):
    from triton_kernels.moe_batch import PackedRoutedExperts, packed_routed_moe
    from dsv2 import ops
    H, I, E = 2048, 1408, 64
    gate_up = (0.02 * torch.randn(E + 2, 2 * I, H, device=dev, generator=g)).to(torch.bfloat16)
    down = (0.02 * torch.randn(E + 2, H, I, device=dev, generator=g)).to(torch.bfloat16)
    x = torch.randn(B, H, device=dev, generator=g).to(torch.bfloat16)
    ids = torch.rand(B, E, device=dev, generator=g).topk(6, dim=-1).indices
    w = torch.rand(B, 6, device=dev, generator=g)
    packed = PackedRoutedExperts(gate_up_weights=gate_up[:E], down_weights=down[:E], hidden_size=H,
                                 intermediate_size=I, num_experts=E, topk=6)
    ref_out = {}

    def ref():
        ref_out["y"] = packed_routed_moe(x, ids, w, packed)
    ids32 = ids.to(torch.int32).contiguous()
    R = 8 * B
    go = torch.zeros(E + 3, dtype=torch.int32, device=dev)
    rt = torch.zeros(R, dtype=torch.int32, device=dev)
    rs, rw = torch.zeros_like(rt), torch.zeros(R, device=dev)
    xs = torch.zeros(R, H, dtype=torch.bfloat16, device=dev)
    h = torch.zeros(R, I, dtype=torch.bfloat16, device=dev)
    y = torch.zeros(B, 8, H, device=dev)
    sync = torch.zeros(E + 4, dtype=torch.int32, device=dev)

    def ours():
        # routed experts only (no shared-expert rows), bucketing + gather + fused MoE
        ops.moe_bucket(ids32, w, 0, E, 0, 0, go, rt, rs, rw, gather_src=x, gather_out=xs)
        ops.moe(gate_up=gate_up, down=down, x_sorted=xs, h=h, group_offsets=go, max_routes_per_group=B,
                route_slot=rs, route_weight=rw, y=y.view(-1, H), sync=sync)
    t_ref = graph_time(ref, iters)
    t_ours = graph_time(ours, iters)
    torch.cuda.synchronize()
    distinct = int((torch.bincount(ids.view(-1), minlength=E) > 0).sum())
    nbytes = distinct * 3 * I * H * 2
    line("moe_routed", t_ref, t_ours, nbytes,
         {"batch": B, "experts_hit": distinct,
          "max_rel_diff": round(relerr(y.sum(1), ref_out["y"].float()), 5)})


def case_linear(name, B, iters, dev, g):
    import triton
    from triton_kernels.attention_decode_batch import _batched_linear_kernel, _select_batched_linear_tile
    from dsv2 import ops
    from dsv2.engine import split_count
    N, K = {"qkva": (3648, 2048), "o": (2048, 2048)}[name]
    w = (0.02 * torch.randn(N, K, device=dev, generator=g)).to(torch.bfloat16)
    x = torch.randn(B, K, device=dev, generator=g).to(torch.bfloat16)
    y_ref = torch.zeros(B, N, dtype=torch.bfloat16, device=dev)
    bb, bo, bk = _select_batched_linear_tile(B)

    def ref():
        _batched_linear_kernel[(triton.cdiv(B, bb), triton.cdiv(N, bo))](
            x, w, y_ref, B, N, K, x.stride(0), x.stride(1), w.stride(0), w.stride(1), y_ref.stride(0),
            y_ref.stride(1), BLOCK_B=bb, BLOCK_O=bo, BLOCK_K=bk, num_warps=4, num_stages=4)
    S = split_count(N, K, torch.cuda.get_device_properties(dev).multi_processor_count)
    part = torch.zeros(S, B, N, device=dev)
    y16 = torch.zeros(B, N, dtype=torch.bfloat16, device=dev)

    def ours_split():
        ops.linear(w=w, n_rows=N, k=K, x=x, y=part[0], epilogue=ops.EPI_STORE_F32, n_tokens=B,
                   family=ops.FAMILY_BATCH, x_group_rows=B, k_splits=S, y_split_stride=part.stride(0))

    def ours_bf16():
        ops.linear(w=w, n_rows=N, k=K, x=x, y=y16, n_tokens=B, family=ops.FAMILY_BATCH, x_group_rows=B)
    t_ref = graph_time(ref, iters)
    t_split = graph_time(ours_split, iters)
    t_bf16 = graph_time(ours_bf16, iters)
    nbytes = N * K * 2
    line(f"{name}_linear", t_ref, t_split, nbytes,
         {"batch": B, "ours": f"tcgen05, fp32 split-K x{S} (as in the decode step)", "ref_tile": [bb, bo, bk],
          "ours_bf16_out_us": round(t_bf16, 2),
          "max_rel_diff": round(relerr(part.sum(0), y_ref.float()), 5)})


def case_attention(B, L, iters, dev, g, ragged_lens=None):
    from triton_kernels.attention_decode_batch import batched_attention_decode_q1_triton
    from dsv2 import ops
    S = (L + 64 + 63) // 64 * 64
    scale = 192 ** -0.5
    # latent cache + absorbed queries (ours), and the equivalent expanded K / V (reference):
    # K[h] = [c W_UK[h]^T | k_pe], V[h] = c W_UV[h]^T, q[h] = [q_nope[h] | q_pe[h]]
    lat = (0.5 * torch.randn(B, S, 576, device=dev, generator=g)).to(torch.bfloat16)
    w_uk = (0.05 * torch.randn(16, 128, 512, device=dev, generator=g)).to(torch.bfloat16)
    w_uv = (0.05 * torch.randn(16, 128, 512, device=dev, generator=g)).to(torch.bfloat16)
    q_nope = (0.5 * torch.randn(B, 16, 128, device=dev, generator=g)).to(torch.bfloat16)
    q_pe = (0.5 * torch.randn(B, 16, 64, device=dev, generator=g)).to(torch.bfloat16)
    k_exp = torch.empty(B, 16, S, 192, dtype=torch.bfloat16, device=dev)
    v_exp = torch.empty(B, 16, S, 128, dtype=torch.bfloat16, device=dev)
    for b0 in range(0, B, 32):
        c = lat[b0:b0 + 32, :, :512].float()
        k_exp[b0:b0 + 32, :, :, :128] = torch.einsum("bsc,hdc->bhsd", c, w_uk.float()).to(torch.bfloat16)
        k_exp[b0:b0 + 32, :, :, 128:] = lat[b0:b0 + 32, None, :, 512:]
        v_exp[b0:b0 + 32] = torch.einsum("bsc,hdc->bhsd", c, w_uv.float()).to(torch.bfloat16)
    q_exp = torch.cat([q_nope, q_pe], -1).view(B, 16, 1, 192).contiguous()
    q_abs = torch.einsum("bhd,hdc->bhc", q_nope.float(), w_uk.float()).to(torch.bfloat16).contiguous()
    pos1 = torch.tensor([L - 1], dtype=torch.int64, device=dev)
    ref_out = {}

    def ref():
        ref_out["o"] = batched_attention_decode_q1_triton(q_exp, k_exp, v_exp, pos1, scale)
    posB = torch.full((B,), L - 1, dtype=torch.int64, device=dev)
    ws = ops.mla_workspace(B, S, 64, dev)
    o_lat = torch.zeros(B, 16, 512, dtype=torch.bfloat16, device=dev)

    def ours():
        ops.mla_decode(q_abs=q_abs, q_pe=q_pe, cache=lat, positions=posB, softmax_scale=scale, split_len=64,
                       o_lat=o_lat, **ws)
    t_ref = graph_time(ref, iters)
    t_ours = graph_time(ours, iters)
    o_ours = torch.einsum("bhc,hdc->bhd", o_lat.float(), w_uv.float())
    ref_bytes = B * L * 16 * (192 + 128) * 2
    our_bytes = B * L * 576 * 2
    line("attention", t_ref, t_ours, our_bytes,
         {"batch": B, "length": L, "ref_bytes": ref_bytes, "ref_GBps": round(ref_bytes / t_ref / 1e3, 1),
          "note": "ref reads the expanded per-head K/V cache (10240 B per token), ours the 1152 B latent row",
          "max_rel_diff": round(relerr(o_ours, ref_out["o"].float().view(B, 16, 128)), 5)})
    if ragged_lens is not None:
        del k_exp, v_exp
        S_r = (max(ragged_lens) + 64 + 63) // 64 * 64
        lat_r = (0.5 * torch.randn(B, S_r, 576, device=dev, generator=g)).to(torch.bfloat16)
        pos_r = torch.tensor(ragged_lens, dtype=torch.int64, device=dev) - 1
        ws_r = ops.mla_workspace(B, S_r, 64, dev)

        def ours_r():
            ops.mla_decode(q_abs=q_abs, q_pe=q_pe, cache=lat_r, positions=pos_r, softmax_scale=scale,
                           split_len=64, o_lat=o_lat, **ws_r)
        t_r = graph_time(ours_r, iters)
        nb = int((pos_r + 1).sum()) * 576 * 2
        print(json.dumps({"case": "attention_ragged_ours_only", "batch": B, "ours_us": round(t_r, 2),
                          "ours_GBps": round(nb / t_r / 1e3, 1), "bytes": nb,
                          "note": "the reference attention takes one shared cache position (no ragged rows)"}),
              flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, default=256)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--cases", default="moe,qkva,o,attention")
    a = ap.parse_args()
    cases = set(a.cases.split(","))
    if not (REF / "triton_kernels").exists():
        print(json.dumps({"unavailable": f"reference kernels not found under {REF}"}))
        return
    sys.path.insert(0, str(REF))
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev).manual_seed(0)
    import bench
    lens = bench.prompt_lengths(bench.CONFIGS[4], a.batch)
    L = int(round(sum(lens) / len(lens)))
    if "moe" in cases:
        case_moe(a.batch, a.iters, dev, g)
        torch.cuda.empty_cache()
    for name in ("qkva", "o"):
        if name in cases:
            case_linear(name, a.batch, a.iters, dev, g)
    if "attention" in cases:
        case_attention(a.batch, L, a.iters, dev, g, ragged_lens=lens)


if __name__ == "__main__":
    main()
