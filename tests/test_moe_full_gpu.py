"""The fused MoE launch at its production shape against the oracle.

64 routed experts + the two halves of the shared MLP (66 groups, intermediate 1408,
hidden 2048, bf16 N(0, 0.02) weights), routed by the library's own router and
bucketing (fp32 gate linear, softmax, top-6, stable counting sort, expert-ordered copy
of the activations), for B in {1, 32, 256}, with uniform routing and with the skewed
router of the long-context workload (a Zipf(1.1) per-expert logit offset, so a few
experts take hundreds of routes: their groups span several token tiles and the work
list is dealt from the global counter).  Checks:
  * routing: top-6 ids bit-exact to the oracle router up to ties within 1e-3, group
    offsets / route lists equal to the oracle's counting sort;
  * every routed and shared slot within 1e-2 (max rel err) of the oracle's per-route
    expert MLP (bf16 rounding points as HF), and the slot sum (= the MoE output) within
    2e-2 of the HF-semantics MoE (oracle.ops.moe, fp32 sums, on the GPU);
  * a second call gives identical bits and leaves the progress counters at zero.
"""
import pytest
import torch

from oracle import ops as O
from oracle.hf_model import router_bias_zipf

pytestmark = pytest.mark.gpu
DEV = "cuda"
E, I, H = 64, 1408, 2048
G = E + 2


def relerr(a, b):
    a, b = a.double(), b.double()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))


@pytest.fixture(scope="module")
def experts():
    g = torch.Generator(device=DEV).manual_seed(77)
    gate_up = (0.02 * torch.randn(G, 2 * I, H, device=DEV, generator=g)).to(torch.bfloat16)
    down = (0.02 * torch.randn(G, H, I, device=DEV, generator=g)).to(torch.bfloat16)
    gate_w = (0.02 * torch.randn(E, H, device=DEV, generator=g)).to(torch.bfloat16)
    return gate_up, down, gate_w


@pytest.mark.parametrize("B,skew", [(1, False), (32, False), (256, False), (32, True), (256, True)])
def test_fused_moe_66_groups_matches_oracle(experts, B, skew):
    from dsv2 import ops as D
    gate_up, down, gate_w = experts
    g = torch.Generator(device=DEV).manual_seed(1000 + B + 7 * skew)
    x = torch.randn(B, H, device=DEV, generator=g).to(torch.bfloat16)
    bias = router_bias_zipf(E, 1.1, seed=4).to(DEV) if skew else None
    R = 8 * B
    buf = {k: torch.zeros(s, dtype=t, device=DEV) for k, s, t in (
        ("logits", (B, E), torch.float32), ("ids32", (B, 6), torch.int32), ("ids64", (B, 6), torch.int64),
        ("tw", (B, 6), torch.float32), ("go", (G + 1,), torch.int32), ("xs", (R, H), torch.bfloat16),
        ("rt", (R,), torch.int32), ("rs", (R,), torch.int32), ("rw", (R,), torch.float32),
        ("h", (R, I), torch.bfloat16), ("sync", (G + 2,), torch.int32))}
    D.router(x=x, w=gate_w, scaling=1.0, bias=bias, logits=buf["logits"], topk_ids32=buf["ids32"],
             topk_weights=buf["tw"], topk_ids64=buf["ids64"], gather_out=buf["xs"], expert_lo=0, n_local=E,
             shared_lo=0, shared_hi=B, group_offsets=buf["go"], route_token=buf["rt"], route_slot=buf["rs"],
             route_weight=buf["rw"])
    outs = []
    for _ in range(2):
        y = torch.zeros(B, 8, H, device=DEV)
        D.moe(gate_up=gate_up, down=down, x_sorted=buf["xs"], h=buf["h"], group_offsets=buf["go"],
              max_routes_per_group=B, route_slot=buf["rs"], route_weight=buf["rw"], y=y.view(-1, H),
              sync=buf["sync"])
        torch.cuda.synchronize()
        outs.append(y)
        assert int(buf["sync"].abs().sum()) == 0
    assert torch.equal(outs[0], outs[1])
    y = outs[0]

    # routing against the oracle router and counting sort
    lg, ids_ref, _ = O.router(x.cpu(), gate_w.cpu(), 1.0, None if bias is None else bias.cpu())
    p = torch.softmax(lg, -1)
    ids = buf["ids64"].cpu()
    for b in range(B):
        got, want = set(ids[b].tolist()), set(ids_ref[b].tolist())
        if got != want:
            vals = p[b, sorted(got ^ want)]
            assert float(vals.max() - vals.min()) <= 1e-3 * float(vals.max()), (b, got, want)
    go, rt, rs, rw = O.bucket(ids, buf["tw"].cpu(), 0, E, 0, B)
    assert torch.equal(buf["go"].cpu(), go)
    n = int(go[-1])
    assert torch.equal(buf["rt"].cpu()[:n], rt) and torch.equal(buf["rs"].cpu()[:n], rs)
    counts = (go[1:E + 1] - go[:E])
    if skew and B == 256:
        assert int(counts.max()) > 128  # a group spanning several 128-token tiles

    # every slot against the oracle's per-route expert MLP (on the GPU, fp32 math)
    y_ref = torch.zeros(B * 8, H, device=DEV)
    for gi in range(G):
        a, c = int(go[gi]), int(go[gi + 1])
        if a == c:
            continue
        xr = x[rt[a:c].long().to(DEV)]
        hr = O.linear(gate_up[gi, :I], xr, "swiglu", up=gate_up[gi, I:])
        y_ref[rs[a:c].long().to(DEV)] = O.linear(down[gi], hr, "scale", scale=rw[a:c].to(DEV))
    assert relerr(y.view(-1, H), y_ref) < 1e-2
    # the combined output against the HF-semantics MoE
    moe_ref = O.moe(x, ids.to(DEV), buf["tw"], gate_up[:E], down[:E],
                    torch.cat([gate_up[E, :I], gate_up[E + 1, :I]]), torch.cat([gate_up[E, I:], gate_up[E + 1, I:]]),
                    torch.cat([down[E], down[E + 1]], 1))
    assert relerr(y.sum(1), moe_ref) < 2e-2
