"""GPU parity of the linear kernels (small family: mma.sync GEMV; batch family: tcgen05
GEMM) against the oracle's fp32 linear for every mode the decode step uses: dense,
batched over heads with strided operands, and grouped (MoE) with device-side route
lists, for each epilogue (bf16, fp32, SwiGLU, route-weight scaling).

Tolerance: max|err| / max|ref| <= 1e-2 (bf16 outputs of fp32 accumulations whose
order differs from the oracle's).
"""
import pytest
import torch

from oracle import ops as O

pytestmark = pytest.mark.gpu
DEV = "cuda"
FAMILIES = ["small", "batch"]


def relerr(a, b):
    a, b = a.double().cpu(), b.double().cpu()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))


@pytest.fixture(scope="module")
def D():
    from dsv2 import ops
    return ops


def fam(D, name):
    return D.FAMILY_SMALL if name == "small" else D.FAMILY_BATCH


def rnd(shape, g, scale=1.0):
    return (torch.randn(*shape, generator=g) * scale).to(torch.bfloat16)


@pytest.mark.parametrize("family", FAMILIES)
@pytest.mark.parametrize("N,K,T", [(3648, 2048, 1), (2048, 2048, 3), (2048, 2048, 8), (3648, 2048, 17),
                                   (2048, 2048, 32), (2048, 2048, 256), (2048, 10944, 5), (300, 512, 300)])
def test_dense(D, family, N, K, T):
    g = torch.Generator().manual_seed(N + K + T)
    w, x = rnd((N, K), g, 0.02), rnd((T, K), g)
    y = torch.zeros(T, N, dtype=torch.bfloat16, device=DEV)
    D.linear(w=w.to(DEV), n_rows=N, k=K, x=x.to(DEV), y=y, family=fam(D, family), n_tokens=T, x_group_rows=T)
    assert relerr(y, O.linear(w, x)) < 1e-2


@pytest.mark.parametrize("family", FAMILIES)
@pytest.mark.parametrize("I,T", [(1408, 1), (1408, 24), (10944, 2), (10944, 64)])
def test_dense_swiglu(D, family, I, T):
    g = torch.Generator().manual_seed(I + T)
    w, x = rnd((2 * I, 2048), g, 0.02), rnd((T, 2048), g)
    y = torch.zeros(T, I, dtype=torch.bfloat16, device=DEV)
    D.linear(w=w.to(DEV), n_rows=I, k=2048, up_offset=I * 2048, x=x.to(DEV), y=y, family=fam(D, family),
             epilogue=D.EPI_SWIGLU, n_tokens=T, w_group_rows=2 * I, x_group_rows=T)
    ref = O.linear(w[:I], x, "swiglu", up=w[I:])
    assert relerr(y, ref) < 1e-2


@pytest.mark.parametrize("family", FAMILIES)
def test_dense_fp32_out(D, family):
    g = torch.Generator().manual_seed(3)
    w, x = rnd((512, 2048), g, 0.02), rnd((4, 2048), g)
    y = torch.zeros(4, 512, device=DEV)
    D.linear(w=w.to(DEV), n_rows=512, k=2048, x=x.to(DEV), y=y, family=fam(D, family), epilogue=D.EPI_STORE_F32,
             n_tokens=4, x_group_rows=4)
    assert relerr(y, O.linear(w, x, "f32")) < 1e-4


@pytest.mark.parametrize("N,K,T,S", [(3648, 2048, 256, 5), (2048, 2048, 256, 9), (2048, 2048, 1, 9),
                                     (3648, 2048, 32, 5), (2048, 10944, 77, 9), (300, 512, 100, 3),
                                     (136, 2048, 255, 2), (2048, 2048, 5, 16), (3648, 2048, 300, 3)])
def test_dense_split_k(D, N, K, T, S):
    """fp32 partials of a K split (the batch decode step's attention projections and dense
    down projection): split s of the K blocks at y[s]; their sum matches the oracle's fp32
    linear, each split matches the oracle over its own K range, and a second call gives the
    same bits.  Up to 256 tokens one CTA takes one (row tile, split) item with its weight
    slice resident (K = 10944: more K blocks than weight slots, streamed); 300 tokens take
    the persistent kernel."""
    g = torch.Generator().manual_seed(N + K + T + S)
    w, x = rnd((N, K), g, 0.02).to(DEV), rnd((T, K), g).to(DEV)
    y = torch.full((S, T, N), float("nan"), device=DEV)
    D.linear(w=w, n_rows=N, k=K, x=x, y=y[0], family=D.FAMILY_BATCH, epilogue=D.EPI_STORE_F32, n_tokens=T,
             x_group_rows=T, k_splits=S, y_split_stride=y.stride(0))
    torch.cuda.synchronize()
    assert not torch.isnan(y).any()
    assert relerr(y.sum(0), O.linear(w.cpu(), x.cpu(), "f32")) < 1e-4
    nkb = K // 64
    for sp in (0, S - 1):
        k0, k1 = sp * nkb // S * 64, (sp + 1) * nkb // S * 64
        ref = O.linear(w[:, k0:k1].cpu(), x[:, k0:k1].cpu(), "f32")
        assert relerr(y[sp], ref) < 1e-4
    y2 = torch.zeros_like(y)
    D.linear(w=w, n_rows=N, k=K, x=x, y=y2[0], family=D.FAMILY_BATCH, epilogue=D.EPI_STORE_F32, n_tokens=T,
             x_group_rows=T, k_splits=S, y_split_stride=y.stride(0))
    assert torch.equal(y, y2)


@pytest.mark.parametrize("family", FAMILIES)
@pytest.mark.parametrize("B", [1, 7, 64])
def test_heads_absorb_and_unabsorb(D, family, B):
    """q_abs[b, h] = q_nope[b, h] @ W_UK[h] (strided q_nope inside qkva) and
    o[b, h] = o_lat[b, h] @ W_UV[h]^T (W_UV a strided view of kv_b)."""
    g = torch.Generator().manual_seed(B)
    qkva = rnd((B, 3648), g)
    kv_b = rnd((4096, 512), g, 0.05)
    w_uk_t = kv_b.view(16, 256, 512)[:, :128].transpose(1, 2).contiguous()
    q_abs = torch.zeros(B, 16, 512, dtype=torch.bfloat16, device=DEV)
    f = fam(D, family)
    qd = qkva.to(DEV)
    D.linear(w=w_uk_t.to(DEV), n_rows=512, k=128, w_row_stride=128, w_group_stride=512 * 128, x=qd,
             x_row_stride=3648, x_group_stride=192, y=q_abs, y_row_stride=16 * 512, y_group_stride=512,
             n_groups=16, n_tokens=B, family=f, w_group_rows=512, x_group_rows=B)
    q_nope = qkva[:, :3072].view(B, 16, 192)[..., :128]
    ref = torch.einsum("bhd,hdc->bhc", q_nope.float(), kv_b.view(16, 256, 512)[:, :128].float())
    assert relerr(q_abs, ref) < 1e-2
    o_lat = rnd((B, 16, 512), g)
    o = torch.zeros(B, 2048, dtype=torch.bfloat16, device=DEV)
    kvd = kv_b.to(DEV)
    D.linear(w=kvd[128:], n_rows=128, k=512, w_row_stride=512, w_group_stride=256 * 512, x=o_lat.to(DEV),
             x_row_stride=16 * 512, x_group_stride=512, y=o, y_row_stride=2048, y_group_stride=128, n_groups=16,
             n_tokens=B, family=f, w_group_rows=128, x_group_rows=B)
    ref = torch.einsum("bhc,hvc->bhv", o_lat.float(), kv_b.view(16, 256, 512)[:, 128:].float()).reshape(B, 2048)
    assert relerr(o, ref) < 1e-2


def _routes(B, n_exp, g):
    ids = torch.stack([torch.randperm(n_exp, generator=g)[:6] for _ in range(B)])
    w = torch.rand(B, 6, generator=g)
    return ids, w


@pytest.mark.parametrize("family", FAMILIES)
@pytest.mark.parametrize("B,bounded", [(1, False), (1, True), (5, True), (32, False), (256, True)])
def test_grouped_moe(D, family, B, bounded):
    """gate_up + SwiGLU and down + route-weight scaling over experts (8 routed + 2 shared
    groups; the expert count is reduced to keep the test small).  bounded: the launch is
    told the total route count, so the small family covers only the groups holding routes."""
    g = torch.Generator().manual_seed(100 + B)
    E, I, H = 8, 1408, 2048
    G = E + 2
    gate_up = rnd((G, 2 * I, H), g, 0.02)
    down = rnd((G, H, I), g, 0.02)
    x = rnd((B, H), g)
    ids, wts = _routes(B, E, g)
    go, rt, rs, rw = O.bucket(ids, wts, 0, E, 0, B)
    R = int(go[-1])
    f = fam(D, family)
    xd, god, rtd, rsd, rwd = x.to(DEV), go.to(DEV), rt.to(DEV), rs.to(DEV), rw.to(DEV)
    h = torch.zeros(R, I, dtype=torch.bfloat16, device=DEV)
    if family == "batch":
        xs = torch.zeros(R, H, dtype=torch.bfloat16, device=DEV)
        D.gather_rows(xd, rtd, god, G, xs, R)
        assert torch.equal(xs.cpu(), x[rt.long()])
        gx, rx = xs, None
    else:
        gx, rx = xd, rtd
    gud, dnd = gate_up.to(DEV), down.to(DEV)
    D.linear(w=gud, n_rows=I, k=H, up_offset=I * H, w_group_stride=2 * I * H, x=gx, y=h, epilogue=D.EPI_SWIGLU,
             n_groups=G, group_offsets=god, max_routes_per_group=B, route_x_row=rx, family=f,
             max_routes=R if bounded else 0,
             w_group_rows=2 * I, x_group_rows=R)
    partial = torch.zeros(B, 8, H, device=DEV)
    D.linear(w=dnd, n_rows=H, k=I, w_group_stride=H * I, x=h, y=partial.view(-1, H), epilogue=D.EPI_SCALE_F32,
             n_groups=G, group_offsets=god, max_routes_per_group=B, route_y_row=rsd, route_scale=rwd, family=f,
             max_routes=R if bounded else 0,
             w_group_rows=H, x_group_rows=R)
    # oracle, route by route
    h_ref = torch.zeros(R, I, dtype=torch.bfloat16)
    p_ref = torch.zeros(B * 8, H)
    for gi in range(G):
        a, b = int(go[gi]), int(go[gi + 1])
        if a == b:
            continue
        xr = x[rt[a:b].long()]
        h_ref[a:b] = O.linear(gate_up[gi, :I], xr, "swiglu", up=gate_up[gi, I:])
        p_ref[rs[a:b].long()] = O.linear(down[gi], h_ref[a:b], "scale", scale=rw[a:b])
    assert relerr(h, h_ref) < 1e-2
    assert relerr(partial.view(-1, H), p_ref) < 1e-2
    if family == "batch":
        # the fused single-launch MoE computes the same values bit for bit, and leaves its
        # progress counters at zero (checked by running it twice)
        sync = torch.zeros(G + 2, dtype=torch.int32, device=DEV)
        for tt in (0, 0, 32):   # auto token tile (twice), and a fixed 32-token tile
            h2 = torch.full((R, I), float("nan"), dtype=torch.bfloat16, device=DEV)
            p2 = torch.zeros(B, 8, H, device=DEV)
            D.moe(gate_up=gud, down=dnd, x_sorted=gx, h=h2, group_offsets=god, max_routes_per_group=B,
                  route_slot=rsd, route_weight=rwd, y=p2.view(-1, H), sync=sync, tile_tokens=tt)
            torch.cuda.synchronize()
            assert torch.equal(h2, h)
            assert torch.equal(p2, partial)
            assert int(sync.abs().sum()) == 0
    # and the combined output equals the HF-semantics MoE
    moe_ref = O.moe(x, ids, wts, gate_up[:E], down[:E], torch.cat([gate_up[E, :I], gate_up[E + 1, :I]]),
                    torch.cat([gate_up[E, I:], gate_up[E + 1, I:]]), torch.cat([down[E], down[E + 1]], 1))
    assert relerr(partial.sum(1), moe_ref) < 2e-2
