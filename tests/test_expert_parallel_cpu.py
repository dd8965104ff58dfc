"""Expert-parallel partition and exchange (dsv2.expert_parallel) on CPU gloo ranks.

Each rank routes its own rows, all-gathers activations / ids / weights with
``gather_routing``, buckets the routes that hit its experts (plus the shared-expert
halves of its own rows) exactly as the engine asks the bucketing kernel to
(expert_lo, n_local, row_lo, row_hi), computes those routes with the oracle's expert
MLP, and ``scatter_sum``s the per-row sums.  Every rank's result must equal the
single-process MoE of its rows.  The GPU path runs the same calls over NCCL.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from dsv2.expert_parallel import ep_shard, gather_routing, scatter_sum
from oracle import ops as O

E, H, I, B_ALL = 8, 64, 32, 12


def _weights():
    g = torch.Generator().manual_seed(3)
    gate_w = torch.randn(E, H, generator=g).to(torch.bfloat16)
    gate_up = (torch.randn(E, 2 * I, H, generator=g) * 0.2).to(torch.bfloat16)
    down = (torch.randn(E, H, I, generator=g) * 0.2).to(torch.bfloat16)
    sh_gate = (torch.randn(2 * I, H, generator=g) * 0.2).to(torch.bfloat16)
    sh_up = (torch.randn(2 * I, H, generator=g) * 0.2).to(torch.bfloat16)
    sh_down = (torch.randn(H, 2 * I, generator=g) * 0.2).to(torch.bfloat16)
    x = torch.randn(B_ALL, H, generator=g).to(torch.bfloat16)
    return gate_w, gate_up, down, sh_gate, sh_up, sh_down, x


def _group_weights(g, shard, gate_up, down, sh_gate, sh_up, sh_down):
    """Weights of group g of this rank: local routed expert, or shared half g - n_local."""
    if g < shard.n_local:
        e = shard.expert_lo + g
        return gate_up[e], down[e]
    s = g - shard.n_local
    rows = slice(s * I, (s + 1) * I)
    return torch.cat([sh_gate[rows], sh_up[rows]], 0), sh_down[:, rows]


def _rank(rank, world, port):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        gate_w, gate_up, down, sh_gate, sh_up, sh_down, x = _weights()
        shard = ep_shard(E, B_ALL, rank, world)
        x_loc = x[shard.row_lo:shard.row_hi].contiguous()
        _, ids_loc, w_loc = O.router(x_loc, gate_w, 1.0)
        ids_all = torch.zeros(B_ALL, 6, dtype=torch.int32)
        w_all = torch.zeros(B_ALL, 6)
        x_all = torch.zeros(B_ALL, H, dtype=torch.bfloat16)
        gather_routing(x_loc, ids_loc.to(torch.int32).contiguous(), w_loc.contiguous(), x_all, ids_all, w_all)
        _, ids_ref, w_ref = O.router(x, gate_w, 1.0)
        assert torch.equal(x_all, x) and torch.equal(ids_all, ids_ref.to(torch.int32)) and torch.equal(w_all, w_ref)
        go, tok, slot, wt = O.bucket(ids_all, w_all, shard.expert_lo, shard.n_local, shard.row_lo, shard.row_hi)
        partial = torch.zeros(B_ALL, 8, H)
        for g in range(shard.n_local + 2):
            gu, dn = _group_weights(g, shard, gate_up, down, sh_gate, sh_up, sh_down)
            for r in range(int(go[g]), int(go[g + 1])):
                b = int(tok[r])
                y = O.expert_mlp(x_all[b:b + 1], gu, dn)[0].float()
                partial.view(-1, H)[int(slot[r])] = y * float(wt[r])
        moe_sum = partial.sum(1)
        out = torch.zeros(shard.rows, H)
        scatter_sum(moe_sum, out)
        ref = O.moe(x, ids_ref, w_ref, gate_up, down, sh_gate, sh_up, sh_down)[shard.row_lo:shard.row_hi]
        err = float((out - ref).abs().max() / ref.abs().max())
        assert err < 1e-2, err
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 4])
def test_expert_parallel_moe_matches_single_process(world):
    mp.start_processes(_rank, args=(world, _free_port()), nprocs=world, start_method="spawn")


def test_shard_partition():
    shards = [ep_shard(64, 256, r, 8) for r in range(8)]
    assert [s.expert_lo for s in shards] == list(range(0, 64, 8)) and all(s.n_local == 8 for s in shards)
    assert [(s.row_lo, s.row_hi) for s in shards] == [(32 * r, 32 * r + 32) for r in range(8)]
    with pytest.raises(ValueError):
        ep_shard(64, 256, 0, 3)
    with pytest.raises(ValueError):
        ep_shard(64, 30, 0, 4)
