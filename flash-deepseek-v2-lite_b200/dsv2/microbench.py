"""Single-kernel timing at decode-step shapes (synthetic data, small device footprint).

    python -m dsv2.microbench --kernel moe_gate_up --batch 256 [--family batch] [--iters 20]

Kernels: moe (fused gate_up + down, batch family), moe_gate_up, moe_down (one MoE layer:
64 routed experts + 2 shared halves, uniform random routing), qkva, absorb, unabsorb, o_proj, dense_gate_up, dense_down,
mla_decode (ctx = --ctx positions per row), router.  Prints one JSON line with the
CUDA-event time per launch and the algorithmic bytes / s.  The footprint of every
case is at most ~1.5 GB, so it can run under `ncu --set full` on one launch.
Run from flash-deepseek-v2-lite_b200/ (or with it on sys.path).
"""
from __future__ import annotations

import argparse
import json
import math

import torch

from . import ops


def _rnd(shape, g, scale=1.0, dev="cuda"):
    return (torch.randn(*shape, generator=g, device=dev) * scale).to(torch.bfloat16)


def _routing(B, n_exp, g, dev):
    scores = torch.rand(B, n_exp, generator=g, device=dev)
    ids = scores.topk(6, dim=-1).indices.to(torch.int32)
    w = torch.rand(B, 6, generator=g, device=dev)
    return ids.contiguous(), w.contiguous()


def build_case(kernel: str, B: int, family: int, ctx: int, split_len: int | None, dev="cuda",
               k_splits: int = 1, tile_tokens: int = 0, ragged: tuple[int, int] | None = None):
    g = torch.Generator(device=dev).manual_seed(0)
    H, I, E = 2048, 1408, 64
    calls = []
    nbytes = 0
    if kernel in ("moe", "moe_gate_up", "moe_down", "router", "router_topk", "moe_bucket"):
        G = E + 2
        gate_up = _rnd((G, 2 * I, H), g, 0.02)
        down = _rnd((G, H, I), g, 0.02)
        x = _rnd((B, H), g)
        gate_w = _rnd((E, H), g, 0.02)
        ids, w = _routing(B, E, g, dev)
        R = 8 * B
        go = torch.zeros(G + 1, dtype=torch.int32, device=dev)
        rt = torch.zeros(R, dtype=torch.int32, device=dev)
        rs = torch.zeros_like(rt)
        rw = torch.zeros(R, device=dev)
        ops.moe_bucket(ids, w, 0, E, 0, B, go, rt, rs, rw)
        xs = torch.zeros(R, H, dtype=torch.bfloat16, device=dev)
        ops.gather_rows(x, rt, go, G, xs, R)
        h = _rnd((R, I), g)
        part = torch.zeros(B, 8, H, device=dev)
        distinct = int((torch.bincount(ids.view(-1).long(), minlength=E) > 0).sum())
        batch = family == ops.FAMILY_BATCH
        if kernel == "moe":
            sync = torch.zeros(G + 2, dtype=torch.int32, device=dev)
            calls.append(lambda: ops.moe(gate_up=gate_up, down=down, x_sorted=xs, h=h, group_offsets=go,
                                         max_routes_per_group=B, route_slot=rs, route_weight=rw,
                                         y=part.view(-1, H), sync=sync, tile_tokens=tile_tokens))
            nbytes = (distinct + 2) * 3 * I * H * 2
        elif kernel == "moe_gate_up":
            calls.append(lambda: ops.linear(
                w=gate_up, n_rows=I, k=H, up_offset=I * H, w_group_stride=2 * I * H, x=xs if batch else x,
                y=h, epilogue=ops.EPI_SWIGLU, n_groups=G, group_offsets=go, max_routes_per_group=B,
                route_x_row=None if batch else rt, family=family, w_group_rows=2 * I, x_group_rows=R,
                max_routes=R))
            nbytes = (distinct + 2) * 2 * I * H * 2
        elif kernel == "moe_down":
            calls.append(lambda: ops.linear(
                w=down, n_rows=H, k=I, w_group_stride=H * I, x=h, y=part.view(-1, H), epilogue=ops.EPI_SCALE_F32,
                n_groups=G, group_offsets=go, max_routes_per_group=B, route_y_row=rs, route_scale=rw,
                family=family, w_group_rows=H, x_group_rows=R, max_routes=R, offsets_prior=True))
            nbytes = (distinct + 2) * H * I * 2
        elif kernel == "moe_bucket":
            calls.append(lambda: ops.moe_bucket(ids, w, 0, E, 0, B, go, rt, rs, rw))
            nbytes = B * 6 * 8
        else:
            logits = torch.zeros(B, E, device=dev)
            i32 = torch.zeros(B, 6, dtype=torch.int32, device=dev)
            i64 = torch.zeros(B, 6, dtype=torch.int64, device=dev)
            tw = torch.zeros(B, 6, device=dev)
            bucket = kernel == "router"
            calls.append(lambda: ops.router(x=x, w=gate_w, scaling=1.0, logits=logits, topk_ids32=i32,
                                            topk_weights=tw, topk_ids64=i64,
                                            gather_out=xs if (bucket and batch) else None, expert_lo=0,
                                            n_local=E, shared_lo=0, shared_hi=B,
                                            group_offsets=go if bucket else None,
                                            route_token=rt, route_slot=rs, route_weight=rw))
            nbytes = E * H * 2 + B * H * 2
    elif kernel in ("qkva", "o_proj", "dense_gate_up", "dense_down"):
        N, K, swiglu = {"qkva": (3648, 2048, False), "o_proj": (2048, 2048, False),
                        "dense_gate_up": (10944, 2048, True), "dense_down": (2048, 10944, False)}[kernel]
        wt = _rnd(((2 if swiglu else 1) * N, K), g, 0.02)
        x = _rnd((B, K), g)
        if k_splits > 1 and not swiglu:
            yp = torch.zeros(k_splits, B, N, device=dev)
            calls.append(lambda: ops.linear(w=wt, n_rows=N, k=K, x=x, y=yp[0], epilogue=ops.EPI_STORE_F32,
                                            n_tokens=B, family=family, x_group_rows=B, k_splits=k_splits,
                                            y_split_stride=yp.stride(0)))
        else:
            y = torch.zeros(B, N, dtype=torch.bfloat16, device=dev)
            calls.append(lambda: ops.linear(w=wt, n_rows=N, k=K, up_offset=N * K if swiglu else 0, x=x, y=y,
                                            epilogue=ops.EPI_SWIGLU if swiglu else ops.EPI_STORE_BF16,
                                            n_tokens=B, family=family, w_group_rows=(2 if swiglu else 1) * N,
                                            x_group_rows=B))
        nbytes = wt.numel() * 2
    elif kernel in ("absorb", "unabsorb"):
        kv_b = _rnd((4096, 512), g, 0.05)
        w_uk_t = kv_b.view(16, 256, 512)[:, :128].transpose(1, 2).contiguous()
        qkva = _rnd((B, 3648), g)
        o_lat = _rnd((B, 16, 512), g)
        q_abs = torch.zeros(B, 16, 512, dtype=torch.bfloat16, device=dev)
        o = torch.zeros(B, 2048, dtype=torch.bfloat16, device=dev)
        if kernel == "absorb":
            calls.append(lambda: ops.linear(w=w_uk_t, n_rows=512, k=128, w_row_stride=128,
                                            w_group_stride=512 * 128, x=qkva, x_row_stride=3648, x_group_stride=192,
                                            y=q_abs, y_row_stride=16 * 512, y_group_stride=512, n_groups=16,
                                            n_tokens=B, family=family, w_group_rows=512, x_group_rows=B))
        else:
            calls.append(lambda: ops.linear(w=kv_b[128:], n_rows=128, k=512, w_row_stride=512,
                                            w_group_stride=256 * 512, x=o_lat, x_row_stride=16 * 512,
                                            x_group_stride=512, y=o, y_row_stride=2048, y_group_stride=128,
                                            n_groups=16, n_tokens=B, family=family, w_group_rows=128,
                                            x_group_rows=B))
        nbytes = 16 * 128 * 512 * 2
    elif kernel == "mla_decode":
        # ctx: fixed length per row; ragged=(lo, hi): lengths uniform in [lo, hi) per row
        hi = ragged[1] if ragged else ctx
        S = hi + 64
        cache = _rnd((B, S, 576), g)
        q_abs = _rnd((B, 16, 512), g, 0.1)
        q_pe = _rnd((B, 16, 64), g, 0.1)
        if ragged:
            gg = torch.Generator().manual_seed(3)
            pos = torch.randint(ragged[0], ragged[1], (B,), generator=gg).to(dev) - 1
        else:
            pos = torch.full((B,), ctx - 1, dtype=torch.int64, device=dev)
        from .engine import choose_split_len
        sl = split_len or choose_split_len(B, S, torch.cuda.get_device_properties(dev).multi_processor_count,
                                           family)
        ws = ops.mla_workspace(B, S, sl, dev, family)
        o_lat = torch.zeros(B, 16, 512, dtype=torch.bfloat16, device=dev)
        calls.append(lambda: ops.mla_decode(q_abs=q_abs, q_pe=q_pe, cache=cache, positions=pos, softmax_scale=0.07,
                                            split_len=sl, o_lat=o_lat, family=family, **ws))
        nbytes = int((pos + 1).sum()) * 576 * 2
    else:
        raise ValueError(kernel)
    return calls, nbytes


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--kernel", required=True)
    ap.add_argument("--batch", type=int, default=256)
    ap.add_argument("--family", default="batch", choices=["small", "batch"])
    ap.add_argument("--ctx", type=int, default=576)
    ap.add_argument("--split-len", type=int, default=None)
    ap.add_argument("--k-splits", type=int, default=1)
    ap.add_argument("--tile-tokens", type=int, default=0, help="moe: tokens per work item (0 = auto)")
    ap.add_argument("--ragged", default=None, help="mla_decode: lo,hi row lengths uniform in [lo, hi)")
    ap.add_argument("--no-graph", action="store_true", help="issue launches from Python (host-bound)")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    a = ap.parse_args()
    fam = ops.FAMILY_BATCH if a.family == "batch" else ops.FAMILY_SMALL
    ragged = tuple(int(v) for v in a.ragged.split(",")) if a.ragged else None
    calls, nbytes = build_case(a.kernel, a.batch, fam, a.ctx, a.split_len, k_splits=a.k_splits,
                               tile_tokens=a.tile_tokens, ragged=ragged)
    for _ in range(a.warmup):
        for c in calls:
            c()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if a.no_graph:
        s.record()
        for _ in range(a.iters):
            for c in calls:
                c()
        e.record()
    else:
        # replay the launches from a CUDA graph (as the decode step does), so the timing
        # is device time, not the host's launch rate
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(a.iters):
                for c in calls:
                    c()
        graph.replay()
        torch.cuda.synchronize()
        s.record()
        graph.replay()
        e.record()
    torch.cuda.synchronize()
    us = s.elapsed_time(e) * 1000 / a.iters
    print(json.dumps({"kernel": a.kernel, "batch": a.batch, "family": a.family, "ctx": a.ragged or a.ctx,
                      "split_len": a.split_len, "us": round(us, 2),
                      "bytes": nbytes, "GBps": round(nbytes / us / 1e3, 1)}))


if __name__ == "__main__":
    main()
