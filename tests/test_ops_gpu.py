"""GPU parity of the elementwise, norm, router and latent-attention kernels against the
oracle (oracle/ops.py) and the reference kernels' golden outputs (tests/golden/).

Tolerances: bf16 outputs of identical fp32 math are compared to 1 bf16 ulp
(rtol 2^-7 plus a small atol); reductions whose order differs from the oracle's
use the stated relative bound on max|err| / max|ref|.
"""
import math

import pytest
import torch

from oracle import ops as O

pytestmark = pytest.mark.gpu

DEV = "cuda"


def relerr(a, b):
    a, b = a.double().cpu(), b.double().cpu()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))


@pytest.fixture(scope="module")
def D():
    from dsv2 import ops
    from dsv2 import _lib
    _lib.load()
    return ops


def test_rmsnorm_matches_reference_golden(D, golden_ref):
    for key in ("rmsnorm_2048", "rmsnorm_512"):
        g = golden_ref[key]
        x, w = g["x"].to(DEV), g["w"].to(DEV)
        y = torch.empty_like(x)
        D.rmsnorm(x, w, g["eps"], y)
        torch.testing.assert_close(y.cpu().float(), g["y"].float(), rtol=2 ** -7, atol=1e-6)
        torch.testing.assert_close(y.cpu().float(), O.rmsnorm(g["x"], g["w"], g["eps"]).float(), rtol=2 ** -7,
                                   atol=1e-6)


def test_rmsnorm_fp32_weight_and_strided_rows(D):
    g = torch.Generator(device="cpu").manual_seed(0)
    x = torch.randn(7, 4096, generator=g).to(torch.bfloat16)
    w = torch.randn(2048, generator=g)
    xs = x.to(DEV)[:, :2048]
    y = torch.empty(7, 2048, dtype=torch.bfloat16, device=DEV)
    D.rmsnorm(xs, w.to(DEV), 1e-6, y)
    torch.testing.assert_close(y.cpu().float(), O.rmsnorm(x[:, :2048], w, 1e-6).float(), rtol=2 ** -7, atol=1e-6)


def test_residual_add_and_silu_mul_golden(D, golden_ref):
    g = golden_ref["residual_add"]
    out = torch.empty_like(g["a"]).to(DEV)
    D.residual_add(g["a"].to(DEV), g["b"].to(DEV), out)
    # bit-exact vs the round-to-nearest oracle; one ulp vs the interpreter's truncated golden
    assert torch.equal(out.cpu(), O.residual_add(g["a"], g["b"]))
    torch.testing.assert_close(out.cpu().float(), g["out"].float(), rtol=2 ** -7, atol=0)
    g = golden_ref["silu_mul"]
    out = torch.empty_like(g["gate"]).to(DEV)
    D.silu_mul(g["gate"].to(DEV), g["up"].to(DEV), out)
    torch.testing.assert_close(out.cpu().float(), g["out"].float(), rtol=2 ** -7, atol=1e-6)


def test_add_rmsnorm_bf16_and_partials(D):
    g = torch.Generator().manual_seed(1)
    B = 5
    h = torch.randn(B, 2048, generator=g).to(torch.bfloat16)
    d = torch.randn(B, 2048, generator=g).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(2048, generator=g)).to(torch.bfloat16)
    hd, yd = h.to(DEV), torch.empty(B, 2048, dtype=torch.bfloat16, device=DEV)
    D.add_rmsnorm(hd, d.to(DEV), w.to(DEV), 1e-6, yd)
    hn, yn = O.add_rmsnorm(h, d, w, 1e-6)
    assert torch.equal(hd.cpu(), hn)
    torch.testing.assert_close(yd.cpu().float(), yn.float(), rtol=2 ** -7, atol=1e-6)
    parts = torch.randn(B, 8, 2048, generator=g)
    hd = h.to(DEV)
    D.add_rmsnorm(hd, parts.to(DEV), w.to(DEV), 1e-6, yd)
    hn, yn = O.add_rmsnorm(h, parts, w, 1e-6)
    torch.testing.assert_close(hd.cpu().float(), hn.float(), rtol=2 ** -7, atol=1e-5)
    torch.testing.assert_close(yd.cpu().float(), yn.float(), rtol=2 ** -6, atol=1e-5)


def test_embed_rmsnorm(D):
    g = torch.Generator().manual_seed(2)
    table = torch.randn(1000, 2048, generator=g).to(torch.bfloat16)
    w = torch.randn(2048, generator=g).to(torch.bfloat16)
    ids = torch.tensor([3, 999, 0, 3], dtype=torch.int64)
    h = torch.empty(4, 2048, dtype=torch.bfloat16, device=DEV)
    y = torch.empty_like(h)
    D.embed_rmsnorm(ids.to(DEV), table.to(DEV), w.to(DEV), 1e-6, h, y)
    assert torch.equal(h.cpu(), table[ids])
    torch.testing.assert_close(y.cpu().float(), O.rmsnorm(table[ids], w, 1e-6).float(), rtol=2 ** -7, atol=1e-6)


def test_prepare_inputs_and_cache_copy_golden(D, golden_ref):
    g = golden_ref["prepare_decode_inputs"]
    B, S = g["batch"], g["attention_mask_index"].numel()
    mask = torch.empty(B, S, dtype=torch.int64, device=DEV)
    pid = torch.empty(B, 1, dtype=torch.int64, device=DEV)
    D.prepare_decode_inputs(g["cache_position"].to(DEV), mask, pid, g["attention_mask_index"].to(DEV), B, S)
    assert torch.equal(mask.cpu(), g["attention_mask"]) and torch.equal(pid.cpu(), g["position_ids"])
    g = golden_ref["copy_single_token_to_cache"]
    dst = g["dst_before"].to(DEV)
    D.copy_token_to_cache(g["src"].to(DEV), dst, g["cache_position"].to(DEV))
    assert torch.equal(dst.cpu(), g["dst_after"])


def _router_case(B, seed, bias=False):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(B, 2048, generator=g).to(torch.bfloat16)
    w = (0.02 * torch.randn(64, 2048, generator=g)).to(torch.bfloat16)
    b = (0.5 * torch.randn(64, generator=g)) if bias else None
    return x, w, b


# B up to 148 places one token per bucketing CTA, 300 three (two warps per token), 700 five
# (one warp per token), 1300 nine (the row-per-warp gather of larger CTAs); without the
# gather, one row is bucketed by the warp that ranks it
@pytest.mark.parametrize("B,gather", [(1, True), (1, False), (3, False), (3, True), (16, True), (17, True),
                                      (64, True), (256, True), (300, True), (700, True), (1300, True)])
def test_router_topk_and_bucketing(D, B, gather):
    x, w, bias = _router_case(B, 10 + B, bias=(B == 17))
    lg, ids, wts = O.router(x, w, 1.0, bias)
    dev = {k: torch.zeros(s, dtype=t, device=DEV) for k, s, t in (
        ("logits", (B, 64), torch.float32), ("ids32", (B, 6), torch.int32), ("ids64", (B, 6), torch.int64),
        ("tw", (B, 6), torch.float32), ("go", (67,), torch.int32), ("xs", (8 * B, 2048), torch.bfloat16),
        ("rt", (8 * B,), torch.int32), ("rs", (8 * B,), torch.int32), ("rw", (8 * B,), torch.float32))}
    xd = x.to(DEV)
    for _ in range(2):  # twice: nothing may depend on state left by the previous call
        D.router(x=xd, w=w.to(DEV), scaling=1.0, bias=None if bias is None else bias.to(DEV),
                 logits=dev["logits"], topk_ids32=dev["ids32"], topk_weights=dev["tw"], topk_ids64=dev["ids64"],
                 gather_out=dev["xs"] if gather else None, expert_lo=0, n_local=64, shared_lo=0, shared_hi=B,
                 group_offsets=dev["go"], route_token=dev["rt"], route_slot=dev["rs"], route_weight=dev["rw"])
    torch.cuda.synchronize()
    torch.testing.assert_close(dev["logits"].cpu(), lg, rtol=1e-4, atol=1e-5)
    got = dev["ids64"].cpu()
    p = torch.softmax(lg, -1)
    for r in range(B):
        if set(got[r].tolist()) != set(ids[r].tolist()):
            # only score ties within 1e-3 (relative) may swap the 6th choice
            diff = set(got[r].tolist()) ^ set(ids[r].tolist())
            vals = p[r, list(diff)]
            assert float(vals.max() - vals.min()) <= 1e-3 * float(vals.max())
    assert torch.equal(dev["ids32"].cpu().long(), got)
    torch.testing.assert_close(dev["tw"].cpu(), torch.gather(p, 1, got), rtol=1e-5, atol=1e-7)
    go, rt, rs, rw = O.bucket(got, dev["tw"].cpu(), 0, 64, 0, B)
    assert torch.equal(dev["go"].cpu(), go)
    n = int(go[-1])
    assert torch.equal(dev["rt"].cpu()[:n], rt) and torch.equal(dev["rs"].cpu()[:n], rs)
    assert torch.equal(dev["rw"].cpu()[:n], rw)
    if gather:
        assert torch.equal(dev["xs"].cpu()[:n], x[rt.long()])  # expert-ordered activation copy


# B up to 256 takes one token group per cluster; 1300 and 4096 loop over groups and need the
# grid barrier with every cluster resident
@pytest.mark.parametrize("B,parts", [(1, 3), (5, 1), (64, 0), (256, 5), (256, -1), (1300, 8), (4096, 3)])
def test_fused_router_equals_add_rmsnorm_then_router(D, B, parts):
    """The single-launch router (residual add + RMSNorm, gate, top-6, bucketing, gather)
    against add_rmsnorm followed by the router and the bucketing launch: the same bits in
    every output.  parts > 0: fp32 split-K partials as delta; -1: a bf16 delta; 0: none."""
    g = torch.Generator().manual_seed(40 + B)
    h0 = torch.randn(B, 2048, generator=g).to(torch.bfloat16).to(DEV)
    if parts > 0:
        delta = (0.3 * torch.randn(B, parts, 2048, generator=g)).to(DEV)
    elif parts < 0:
        delta = (0.3 * torch.randn(B, 2048, generator=g)).to(torch.bfloat16).to(DEV)
    else:
        delta = None
    nw = (1 + 0.1 * torch.randn(2048, generator=g)).to(torch.bfloat16).to(DEV)
    w = (0.02 * torch.randn(64, 2048, generator=g)).to(torch.bfloat16).to(DEV)
    bias = (0.5 * torch.randn(64, generator=g)).to(DEV) if B == 256 else None

    def bufs():
        return {k: torch.full(sh, -7, dtype=t, device=DEV) for k, sh, t in (
            ("logits", (B, 64), torch.float32), ("ids32", (B, 6), torch.int32), ("ids64", (B, 6), torch.int64),
            ("tw", (B, 6), torch.float32), ("go", (67,), torch.int32), ("xs", (8 * B, 2048), torch.bfloat16),
            ("rt", (8 * B,), torch.int32), ("rs", (8 * B,), torch.int32), ("rw", (8 * B,), torch.float32),
            ("x", (B, 2048), torch.bfloat16))}
    # reference: two launches of add_rmsnorm + router with bucketing in its own launch
    ha, ra = h0.clone(), bufs()
    D.add_rmsnorm(ha, delta, nw, 1e-6, ra["x"])
    D.router(x=ra["x"], w=w, scaling=1.5, bias=bias, logits=ra["logits"], topk_ids32=ra["ids32"],
             topk_weights=ra["tw"], topk_ids64=ra["ids64"], gather_out=ra["xs"], expert_lo=0, n_local=64,
             shared_lo=0, shared_hi=B, group_offsets=ra["go"], route_token=ra["rt"], route_slot=ra["rs"],
             route_weight=ra["rw"])
    # one launch, twice (the grid barrier's counters carry over between launches)
    sync = torch.zeros(2, dtype=torch.int32, device=DEV)
    from dsv2 import _lib
    for _ in range(2):
        hb, rb = h0.clone(), bufs()
        n0 = _lib.kernel_launches()
        D.router(x=rb["x"], w=w, scaling=1.5, bias=bias, logits=rb["logits"], topk_ids32=rb["ids32"],
                 topk_weights=rb["tw"], topk_ids64=rb["ids64"], gather_out=rb["xs"], expert_lo=0, n_local=64,
                 shared_lo=0, shared_hi=B, group_offsets=rb["go"], route_token=rb["rt"], route_slot=rb["rs"],
                 route_weight=rb["rw"], residual=hb, delta=delta, norm_w=nw, eps=1e-6, sync=sync)
        if B <= 1300:
            assert _lib.kernel_launches() - n0 == 1
        torch.cuda.synchronize()
        assert torch.equal(hb, ha)
        for k in ra:
            assert torch.equal(rb[k], ra[k]), k
        assert int(sync[0]) == 0
    assert _lib.device_error(clear=True) == 0
    # and the routing itself against the oracle on that input
    lg, ids, _ = O.router(ra["x"].cpu(), w.cpu(), 1.5, None if bias is None else bias.cpu())
    p = torch.softmax(lg, -1)
    got = rb["ids64"].cpu()
    for r in range(B):
        if set(got[r].tolist()) != set(ids[r].tolist()):
            vals = p[r, sorted(set(got[r].tolist()) ^ set(ids[r].tolist()))]
            assert float(vals.max() - vals.min()) <= 1e-3 * float(vals.max())


def test_router_golden_topk6(D, golden_ref):
    g = golden_ref["router_topk6"]
    lg = g["logits"].to(DEV)
    ids64 = torch.zeros(8, 6, dtype=torch.int64, device=DEV)
    ids32 = torch.zeros(8, 6, dtype=torch.int32, device=DEV)
    tw = torch.zeros(8, 6, device=DEV)
    D.softmax_topk(lg, g["scaling"], ids64, ids32, tw)
    assert torch.equal(ids64.cpu(), g["ids"])
    torch.testing.assert_close(tw.cpu(), g["weights"], rtol=1e-5, atol=1e-7)
    oi, ow = O.softmax_topk6(g["logits"], g["scaling"])
    assert torch.equal(oi, g["ids"])


def test_moe_bucket_expert_parallel_slice(D):
    g = torch.Generator().manual_seed(7)
    B = 40
    ids = torch.stack([torch.randperm(64, generator=g)[:6] for _ in range(B)]).int()
    tw = torch.rand(B, 6, generator=g)
    go = torch.zeros(16 + 3, dtype=torch.int32, device=DEV)
    rt = torch.zeros(8 * B, dtype=torch.int32, device=DEV)
    rs, rw = torch.zeros_like(rt), torch.zeros(8 * B, device=DEV)
    xsrc = torch.randn(B, 2048, generator=g).to(torch.bfloat16)
    xs = torch.zeros(8 * B, 2048, dtype=torch.bfloat16, device=DEV)
    D.moe_bucket(ids.to(DEV), tw.to(DEV), 16, 16, 10, 20, go, rt, rs, rw, gather_src=xsrc.to(DEV), gather_out=xs)
    eg, et, es, ew = O.bucket(ids, tw, 16, 16, 10, 20)
    assert torch.equal(go.cpu(), eg)
    n = int(eg[-1])
    assert torch.equal(rt.cpu()[:n], et) and torch.equal(rs.cpu()[:n], es) and torch.equal(rw.cpu()[:n], ew)
    assert torch.equal(xs.cpu()[:n], xsrc[et.long()])


def _mla_inputs(B, S, lengths, seed):
    g = torch.Generator().manual_seed(seed)
    cache = (torch.randn(B, S, 576, generator=g)).to(torch.bfloat16)
    q_abs = (0.1 * torch.randn(B, 16, 512, generator=g)).to(torch.bfloat16)
    q_pe = (0.1 * torch.randn(B, 16, 64, generator=g)).to(torch.bfloat16)
    pos = torch.tensor(lengths, dtype=torch.int64) - 1
    return cache, q_abs, q_pe, pos


def _short_rows(n, hi, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(1, hi + 1, (n,), generator=g).tolist()


@pytest.mark.parametrize("B,S,lengths,split", [
    (1, 128, [1], 32), (1, 700, [613], 64), (3, 300, [5, 300, 129], 128), (4, 1100, [1100, 64, 65, 700], 32),
    (2, 8300, [8292, 4000], 64),
    (1, 9000, [8999], 32),                  # one row cut into ~150 CTA ranges, one merge of all of them
    (200, 64, _short_rows(200, 64, 1), 32),  # many whole rows per CTA, boundaries inside rows
    (5, 100, [0, 37, 100, 1, 64], 32),      # a row with nothing to attend gives zeros
    (64, 1200, _short_rows(64, 1200, 2), 64)])
def test_mla_decode_vs_oracle(D, B, S, lengths, split):
    """Balanced latent attention (tile stream spread over the SMs, in-launch merge of rows
    cut between CTAs) against the float64 oracle."""
    cache, q_abs, q_pe, pos = _mla_inputs(B, S, lengths, seed=S + B)
    scale = 192 ** -0.5
    ws = D.mla_workspace(B, S, split, DEV)
    o_lat = torch.full((B, 16, 512), float("nan"), dtype=torch.bfloat16, device=DEV)
    args = dict(q_abs=q_abs.to(DEV), q_pe=q_pe.to(DEV), cache=cache.to(DEV), positions=pos.to(DEV),
                softmax_scale=scale, split_len=split)
    D.mla_decode(o_lat=o_lat, **args, **ws)
    ref = O.mla_decode(q_abs, q_pe, cache, pos + 1, scale)
    # bf16 P (as the reference's P.V) and bf16 output: 1e-2 relative bound
    assert not torch.isnan(o_lat.float()).any()
    assert relerr(o_lat.cpu(), ref) < 1e-2
    # the row tickets are left at zero, and a second call gives the same bits
    assert int(ws["row_sync"].abs().sum()) == 0
    o2 = torch.zeros_like(o_lat)
    D.mla_decode(o_lat=o2, **args, **ws)
    torch.cuda.synchronize()
    assert torch.equal(o2, o_lat)
    assert int(ws["row_sync"].abs().sum()) == 0


@pytest.mark.parametrize("S,L,split", [(128, 1, 32), (128, 33, 32), (700, 613, 64), (1200, 1100, 64),
                                        (9000, 8999, 64)])
def test_mla_deferred_merge_into_unabsorb(D, S, L, split):
    """One row: the attention leaves its partials unmerged (part_count) and the un-absorb
    GEMV merges them while loading its activations.  Against the usual pair (in-launch merge
    into o_lat, then the GEMV over o_lat): same tolerance as the GEMV tests, twice in a row,
    and the first/count record names CTAs that hold tiles."""
    cache, q_abs, q_pe, pos = _mla_inputs(1, S, [L], seed=S + L)
    g = torch.Generator().manual_seed(L)
    kv_b = (torch.randn(4096, 512, generator=g) * 0.05).to(torch.bfloat16).to(DEV)
    scale = 192 ** -0.5
    ws = D.mla_workspace(1, S, split, DEV)
    args = dict(q_abs=q_abs.to(DEV), q_pe=q_pe.to(DEV), cache=cache.to(DEV), positions=pos.to(DEV),
                softmax_scale=scale, split_len=split)
    lin = dict(w=kv_b[128:], n_rows=128, k=512, w_row_stride=512, w_group_stride=256 * 512,
               x_row_stride=16 * 512, x_group_stride=512, y_row_stride=2048, y_group_stride=128, n_groups=16,
               n_tokens=1, family=D.FAMILY_SMALL, w_group_rows=128, x_group_rows=1)
    o_lat = torch.zeros((1, 16, 512), dtype=torch.bfloat16, device=DEV)
    D.mla_decode(o_lat=o_lat, **args, **ws)
    o_ref = torch.zeros(1, 2048, dtype=torch.bfloat16, device=DEV)
    D.linear(x=o_lat, y=o_ref, **lin)
    parts = torch.full((2,), -1, dtype=torch.int32, device=DEV)
    outs = []
    for _ in range(2):
        o_untouched = torch.full((1, 16, 512), float("nan"), dtype=torch.bfloat16, device=DEV)
        D.mla_decode(o_lat=o_untouched, part_count=parts, **args, **ws)
        o = torch.full((1, 2048), float("nan"), dtype=torch.bfloat16, device=DEV)
        D.linear(x=None, y=o, x_parts=(ws["o_part"], ws["ml_part"], parts), **lin)
        torch.cuda.synchronize()
        assert torch.isnan(o_untouched.float()).all()   # o_lat is not written
        assert not torch.isnan(o.float()).any()
        assert relerr(o, o_ref) < 1e-2
        outs.append(o)
    assert torch.equal(outs[0], outs[1])
    first, count = (int(v) for v in parts.cpu())
    tiles = (L + 31) // 32
    assert first >= 0 and 1 <= count <= tiles
    assert int(ws["row_sync"].abs().sum()) == 0


def test_mla_decode_requires_row_tickets(D):
    B, S = 2, 64
    z = torch.zeros(B, 16, 512, dtype=torch.bfloat16, device=DEV)
    ws = D.mla_workspace(B, S, 32, DEV)
    ws.pop("row_sync")
    with pytest.raises(ValueError):
        D.mla_decode(q_abs=z, q_pe=torch.zeros(B, 16, 64, dtype=torch.bfloat16, device=DEV),
                     cache=torch.zeros(B, S, 576, dtype=torch.bfloat16, device=DEV),
                     positions=torch.zeros(B, dtype=torch.int64, device=DEV), softmax_scale=0.1, split_len=32,
                     o_lat=z, **ws)


@pytest.mark.parametrize("B,S,lengths,split", [
    (1, 128, [1], 128), (1, 700, [613], 128), (3, 300, [5, 300, 129], 128), (4, 1100, [1100, 64, 65, 700], 256),
    (5, 256, [128, 129, 256, 1, 200], 256), (2, 8300, [8292, 4000], 1024), (2, 640, [640, 639], 640)])
def test_mla_decode_tcgen05_vs_oracle(D, B, S, lengths, split):
    """Batch-family latent attention on the tensor cores (128-position tiles)."""
    cache, q_abs, q_pe, pos = _mla_inputs(B, S, lengths, seed=S + 7 * B)
    scale = 192 ** -0.5
    n_splits = math.ceil(S / split)
    o_part = torch.zeros(B, n_splits, 16, 512, device=DEV)
    ml = torch.zeros(B, n_splits, 16, 2, device=DEV)
    o_tc = torch.zeros(B, 16, 512, dtype=torch.bfloat16, device=DEV)
    D.mla_decode(q_abs=q_abs.to(DEV), q_pe=q_pe.to(DEV), cache=cache.to(DEV), positions=pos.to(DEV),
                 softmax_scale=scale, split_len=split, o_part=o_part, ml_part=ml, o_lat=o_tc, family=D.FAMILY_BATCH)
    ref = O.mla_decode(q_abs, q_pe, cache, pos + 1, scale)
    assert relerr(o_tc.cpu(), ref) < 1e-2
    # the cache is only read
    assert torch.equal(cache.to(DEV).cpu(), cache)


def test_mla_decode_matches_reference_expanded_attention(D, golden_ref):
    """The absorbed kernel reproduces the reference's expanded-cache attention when the
    expanded K/V are built from a latent cache through W_UK / W_UV."""
    g = torch.Generator().manual_seed(5)
    B, S, L = 2, 80, 71
    cache = torch.randn(B, S, 576, generator=g).to(torch.bfloat16)
    w_uk = (0.05 * torch.randn(16, 128, 512, generator=g))
    w_uv = (0.05 * torch.randn(16, 128, 512, generator=g))
    q_nope = torch.randn(B, 16, 128, generator=g)
    q_pe = torch.randn(B, 16, 64, generator=g).to(torch.bfloat16)
    k_nope = torch.einsum("hdc,bsc->bhsd", w_uk, cache[..., :512].float())
    k = torch.cat([k_nope, cache[:, None, :, 512:].float().expand(B, 16, S, 64)], -1)
    v = torch.einsum("hvc,bsc->bhsv", w_uv, cache[..., :512].float())
    q = torch.cat([q_nope, q_pe.float()], -1)
    scale = 192 ** -0.5
    ref = O.expanded_attention_decode(q, k, v, [L] * B, scale)
    q_abs = torch.einsum("bhd,hdc->bhc", q_nope, w_uk).to(torch.bfloat16).contiguous()
    o_lat = torch.zeros(B, 16, 512, dtype=torch.bfloat16, device=DEV)
    D.mla_decode(q_abs=q_abs.to(DEV), q_pe=q_pe.to(DEV), cache=cache.to(DEV),
                 positions=torch.tensor([L - 1], device=DEV), softmax_scale=scale, split_len=64,
                 o_lat=o_lat, **D.mla_workspace(B, S, 64, DEV))
    out = torch.einsum("bhc,hvc->bhv", o_lat.cpu().float(), w_uv)
    assert relerr(out, ref) < 2e-2
    # and the oracle's expanded attention agrees with the reference kernel's golden output
    gg = golden_ref["batched_attention"]
    n = int(gg["cache_position"]) + 1
    eo = O.expanded_attention_decode(gg["q"][:, :, 0], gg["k"], gg["v"], [n] * gg["q"].shape[0], gg["scale"])
    assert relerr(gg["out"][:, :, 0], eo) < 1e-2


def test_mla_prep_vs_oracle(D, golden_ref):
    g = torch.Generator().manual_seed(9)
    B, S = 3, 50
    qkva = torch.randn(B, 3648, generator=g).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(512, generator=g)).to(torch.bfloat16)
    inv = 1.0 / (10000 ** (torch.arange(0, 64, 2).float() / 64))
    fr = torch.arange(S).float()[:, None] * inv[None, :]
    cos, sin = fr.cos(), fr.sin()
    pos = torch.tensor([0, 17, 49])
    cache = torch.zeros(B, S, 576, dtype=torch.bfloat16, device=DEV)
    q_pe = torch.zeros(B, 16, 64, dtype=torch.bfloat16, device=DEV)
    D.mla_prep(qkva=qkva.to(DEV), kv_norm_w=w.to(DEV), eps=1e-6, cos=cos.to(DEV), sin=sin.to(DEV),
               positions=pos.to(DEV), cache=cache, q_pe_out=q_pe)
    for b in range(B):
        p = int(pos[b])
        row = O.latent_row(qkva[b, 3072:], w, 1e-6, cos[p], sin[p])
        torch.testing.assert_close(cache[b, p].cpu().float(), row.float(), rtol=2 ** -7, atol=1e-6)
        qp = O.rope_interleaved(qkva[b, :3072].view(16, 192)[:, 128:], cos[p], sin[p])
        torch.testing.assert_close(q_pe[b].cpu().float(), qp.float(), rtol=2 ** -7, atol=1e-6)
    # the interleaved rotation equals the reference kernel's half-split RoPE up to the pair order
    gg = golden_ref["build_qkv_rope"]
    p = int(gg["position"])
    c, s = gg["cos"][p, :32], gg["sin"][p, :32]
    hs = O.rope_half_split(gg["q_proj"][:, 128:], c, s)
    torch.testing.assert_close(hs.float(), gg["q_out"][:, 128:].float(), rtol=2 ** -7, atol=1e-6)
    torch.testing.assert_close(O.rope_half_split(gg["k_pe"], c, s).float(), gg["k_new"][0, 128:].float(),
                               rtol=2 ** -7, atol=1e-6)


def test_sum_partials_fixed_order(D):
    g = torch.Generator().manual_seed(9)
    part = torch.randn(6, 8, 2048, generator=g)
    ref = torch.zeros(6, 2048)
    for p in range(5):          # sum the first five slots in slot order
        ref += part[:, p]
    out32 = torch.empty(6, 2048, device=DEV)
    D.sum_partials(part.to(DEV)[:, :5], out32)
    assert torch.equal(out32.cpu(), ref)
    out16 = torch.empty(6, 2048, dtype=torch.bfloat16, device=DEV)
    D.sum_partials(part.to(DEV)[:, :5], out16)
    assert torch.equal(out16.cpu(), ref.to(torch.bfloat16))


@pytest.mark.parametrize("family", ["small", "batch"])
@pytest.mark.parametrize("V,T", [(3001, 1), (5000, 5), (102400, 33)])
def test_lm_head_argmax(D, family, V, T):
    """Greedy token of bf16 logits without materialising them: the chosen index holds the
    largest bf16 logit (oracle fp32 product rounded to bf16), lowest index among equals
    whose value the oracle reproduces; input_ids / positions are updated in place."""
    g = torch.Generator().manual_seed(V + T)
    w = (torch.randn(V, 2048, generator=g) * 0.02).to(torch.bfloat16)
    x = torch.randn(T, 2048, generator=g).to(torch.bfloat16)
    keys = torch.zeros(((V + 15) // 16) * T, dtype=torch.int64, device=DEV)
    nxt = torch.full((T,), -1, dtype=torch.int64, device=DEV)
    inp = torch.full((T,), -1, dtype=torch.int64, device=DEV)
    pos = torch.arange(T, dtype=torch.int64, device=DEV) * 3
    f = D.FAMILY_SMALL if family == "small" else D.FAMILY_BATCH
    D.lm_head_argmax(w=w.to(DEV), x=x.to(DEV), keys=keys, next_ids=nxt, family=f, input_ids=inp, positions=pos)
    logits = (x.float() @ w.float().t()).to(torch.bfloat16).float()
    got = nxt.cpu()
    best = logits.max(dim=1).values
    picked = logits[torch.arange(T), got]
    # the pick is a maximal bf16 logit up to one ulp of summation-order difference
    assert bool(((best - picked) <= best.abs() * 2 ** -7).all())
    ref = logits.argmax(dim=1)
    # with a unique maximum (all rows here) the index is the reference's
    uniq = (logits == best[:, None]).sum(1) == 1
    agree = (got == ref) | ~uniq
    assert float(agree.float().mean()) >= 0.95
    assert torch.equal(inp.cpu(), got)
    assert torch.equal(pos.cpu(), torch.arange(T) * 3 + 1)
