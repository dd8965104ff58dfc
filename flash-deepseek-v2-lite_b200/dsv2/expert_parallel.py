"""Expert-parallel (EP) partition and exchange of the MoE layers across ranks.

One process per GPU.  With N ranks:
  * rank r owns the routed experts [64 r / N, 64 (r + 1) / N) and the batch rows
    [B r / N, B (r + 1) / N) (attention is data parallel: each rank keeps its rows'
    latent cache); every other weight is replicated;
  * per MoE layer each rank routes its own rows, then ``gather_routing`` all-gathers the
    normalised activations [B/N, 2048] bf16, the top-6 ids [B/N, 6] int32 and weights
    [B/N, 6] fp32 into [B, ...] buffers (rank order = row order);
  * each rank buckets the routes of all B rows that hit its experts, plus the two
    shared-expert halves of its own rows only, and runs the grouped GEMMs;
  * the per-row fp32 sums of its slots are reduce-scattered (``scatter_sum``) so every
    rank receives the full MoE output of its own rows.
The reference runs one GPU and has no expert parallelism (pack_routed_experts rejects
ep_size != 1, moe_batch.py:325-326).

The functions take any torch.distributed process group: NCCL on the GPUs (captured in
the decode step's CUDA graph), gloo for the CPU tests of the partition and exchange.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class EpShard:
    rank: int
    world: int
    n_experts: int
    rows: int            # batch rows owned by this rank

    @property
    def n_local(self) -> int:
        return self.n_experts // self.world

    @property
    def expert_lo(self) -> int:
        return self.rank * self.n_local

    @property
    def row_lo(self) -> int:
        """First row of this rank in the gathered [B, ...] buffers."""
        return self.rank * self.rows

    @property
    def row_hi(self) -> int:
        return self.row_lo + self.rows


def ep_shard(n_experts: int, batch_all: int, rank: int, world: int) -> EpShard:
    """Partition of experts and rows for `rank` of `world`; both must divide evenly."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    if n_experts % world:
        raise ValueError(f"{n_experts} experts do not divide over {world} ranks")
    if batch_all % world:
        raise ValueError(f"batch {batch_all} does not divide over {world} ranks")
    return EpShard(rank=rank, world=world, n_experts=n_experts, rows=batch_all // world)


def gather_routing(x: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor, x_all: torch.Tensor,
                   ids_all: torch.Tensor, weights_all: torch.Tensor, group=None) -> None:
    """All-gather this rank's activations / top-6 ids / weights into the [B, ...] buffers."""
    import torch.distributed as dist
    dist.all_gather_into_tensor(x_all, x, group=group)
    dist.all_gather_into_tensor(ids_all, ids, group=group)
    dist.all_gather_into_tensor(weights_all, weights, group=group)


def scatter_sum(moe_sum: torch.Tensor, out_local: torch.Tensor, group=None) -> None:
    """Sum the [B, 2048] per-rank expert outputs over ranks; this rank receives its rows."""
    import torch.distributed as dist
    dist.reduce_scatter_tensor(out_local, moe_sum, group=group)
