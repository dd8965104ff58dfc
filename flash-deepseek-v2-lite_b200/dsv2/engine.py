"""Decode engine: HF DeepSeek-V2 model + latent KV cache + CUDA-graph q_len=1 decode.

Mirrors the reference runner (src/run.py):
  * the HF model object stays the source of weights and runs the eager prefill
    (src/run.py:526-544);
  * one q_len = 1 decode step over all layers is captured in a torch.cuda.CUDAGraph
    and replayed (src/run.py:591-688), after warm-up steps whose effects are rolled
    back (src/run.py:641-656);
  * --kernel-family small | batch selects the GEMV or the tcgen05 linear kernels
    (src/run.py:53-64).
Differences by design: the cache is the 576-wide latent cache [L, B, S, 576] with
per-row positions (ragged batches), the residual add is fused into the following
RMSNorm, and the two shared experts run inside the grouped MoE launch.  With
world > 1 the routed experts are sharded across ranks (expert parallel) and the
batch rows across ranks (attention data parallel); the MoE activations are
all-gathered and the expert outputs reduce-scattered with NCCL inside the graph.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from . import ops
from .expert_parallel import ep_shard, gather_routing, scatter_sum
from .model import (HIDDEN, KV_LORA, LATENT_ROW, N_HEADS, QK_NOPE, QKVA_ROWS, Q_DIM, SLOTS, TOPK,
                    V_DIM, LayerPack, check_config, pack_layer, rope_tables)

FAMILIES = {"small": ops.FAMILY_SMALL, "batch": ops.FAMILY_BATCH}


def choose_split_len(batch: int, max_len: int, num_sms: int, family: int = ops.FAMILY_SMALL) -> int:
    """split_len of mla_decode.  FAMILY_SMALL (balanced kernel): the fewest positions a CTA
    takes, 64 (two tiles), so that short contexts use fewer CTAs and merge fewer partials.
    FAMILY_BATCH (tcgen05 split grid): large batches use 256-position splits, smaller
    batches about four CTAs per SM; multiples of 64 positions."""
    if family == ops.FAMILY_SMALL:
        return 64
    unit = 64
    if batch * 2 >= 3 * num_sms:
        return int(min(256, (max_len + unit - 1) // unit * unit))
    s = math.ceil(batch * max_len / (4 * num_sms))
    s = (s + unit - 1) // unit * unit
    return int(min(max(s, unit), 4096))


def split_count(n_rows: int, k: int, num_sms: int, n_tokens: int = 256) -> int:
    """K splits for a dense batch-family linear with fp32 partial outputs.  Decode batches
    (<= 256 tokens: one (row tile, split) item per CTA, weights requested before the
    programmatic-launch wait): as many splits as fill the SMs (up to 5), so each CTA's
    weight slice and activation traffic are small.  Larger token batches (kernel prefill, persistent
    kernel over several token tiles): about one 128-row tile per two SMs, which also keeps
    the partials the consumer sums few.  At least one 64-wide K block per split, at most 16."""
    m_tiles = (n_rows + 127) // 128
    if n_tokens <= 256:
        # at most 5: the consumers (mla_prep, the fused add + RMSNorm) read every partial
        # (measured on B200, config 4: o_proj 5 splits 8.11 ms/step vs 9 splits 8.14-8.16)
        s = max(1, num_sms // m_tiles)
        return int(min(s, k // 64, 5))
    s = max(1, round(num_sms / (2 * m_tiles)))
    return int(min(s, max(1, (k // 64) // 2), 16))


@dataclass
class DecodeState:
    positions: torch.Tensor   # [B] int64: write position of the next token
    input_ids: torch.Tensor   # [B] int64: token fed to the next step


class _CudaArray:
    """__cuda_array_interface__ over a raw device pointer (zero-copy torch view)."""

    def __init__(self, ptr: int, shape: tuple, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 3}


def _device_view(ptr: int, shape: tuple, dtype: torch.dtype, dev: torch.device) -> torch.Tensor:
    typestr = {torch.int16: "<i2", torch.int32: "<i4", torch.float32: "<f4"}[dtype]
    with torch.cuda.device(dev):
        return torch.as_tensor(_CudaArray(ptr, shape, typestr), device=dev)


class DecodeEngine:
    def __init__(self, model, batch: int, max_len: int, family: str = "batch", *,
                 rank: int = 0, world: int = 1, group=None, gate_bias: torch.Tensor | None = None,
                 alias_hf: bool = True, fused_moe: bool = True, keep_logits: bool = False,
                 cache: torch.Tensor | None = None):
        cfg = model.config
        check_config(cfg)
        if family not in FAMILIES:
            raise ValueError(f"Unknown kernel family: {family}")
        self.model = model
        self.cfg = cfg
        self.family_name = family
        self.family = FAMILIES[family]
        self.dev = model.lm_head.weight.device
        self.B = int(batch)                  # rows owned by this rank
        self.max_len = int(max_len)
        self.rank, self.world, self.group = rank, world, group
        self.fused_moe = fused_moe
        # B = 1, small family: the un-absorb GEMV merges the attention's partials (spread over
        # its CTAs) instead of one attention CTA
        self.defer_mla_merge = True
        self._gate_bias = gate_bias
        self.keep_logits = keep_logits   # also materialise the bf16 logits every step
        # cache given: rows of this engine are tokens of the cache's sequences (kernel
        # prefill); cache_rows[b] names the sequence of row b
        self._external_cache = cache
        self.B_all = self.B * world
        self.shard = ep_shard(int(cfg.n_routed_experts), self.B_all, rank, world)
        self.n_local = self.shard.n_local
        self.expert_lo = self.shard.expert_lo
        self.layers: list[LayerPack] = [
            pack_layer(l, self.expert_lo, self.n_local, alias_hf=alias_hf and world == 1, gate_bias=gate_bias)
            for l in model.model.layers
        ]
        self.L = len(self.layers)
        self.embed = model.model.embed_tokens.weight.detach()
        self.final_norm_w = model.model.norm.weight.detach()
        self.final_eps = float(model.model.norm.variance_epsilon)
        self.lm_head = model.lm_head.weight.detach()
        self.vocab = int(self.lm_head.shape[0])
        self.scale = float(model.model.layers[0].self_attn.scaling)
        self.cos, self.sin = rope_tables(model, self.max_len, self.dev)
        props = torch.cuda.get_device_properties(self.dev)
        self.num_sms = props.multi_processor_count
        self.split_len = choose_split_len(self.B, self.max_len, self.num_sms)
        self.n_splits = ops.mla_splits(self.B, self.max_len, self.split_len, self.num_sms)
        self._alloc()
        self.graph = None
        self._saved = None

    # ------------------------------------------------------------------ buffers
    def _alloc(self):
        B, dev, bf = self.B, self.dev, torch.bfloat16
        f32, i32, i64 = torch.float32, torch.int32, torch.int64
        if self._external_cache is not None:
            self.cache = self._external_cache
            self.cache_rows = torch.zeros(B, device=dev, dtype=i32)
        else:
            self.cache = torch.zeros((self.L, B, self.max_len, LATENT_ROW), device=dev, dtype=bf)
            self.cache_rows = None
        self.positions = torch.zeros(B, device=dev, dtype=i64)
        self.input_ids = torch.zeros(B, device=dev, dtype=i64)
        self.next_ids = torch.zeros(B, device=dev, dtype=i64)
        self.h = torch.zeros((B, HIDDEN), device=dev, dtype=bf)
        self.x = torch.zeros((B, HIDDEN), device=dev, dtype=bf)
        self.qkva = torch.zeros((B, QKVA_ROWS), device=dev, dtype=bf)
        self.q_pe = torch.zeros((B, N_HEADS, 64), device=dev, dtype=bf)
        self.q_nope = torch.zeros((B, N_HEADS, QK_NOPE), device=dev, dtype=bf)
        # batch family: split-K fp32 partials for the dense linears whose consumers sum them
        self.split_k = self.family == ops.FAMILY_BATCH
        if self.split_k:
            s_q = split_count(QKVA_ROWS, HIDDEN, self.num_sms, B)
            s_o = split_count(HIDDEN, N_HEADS * V_DIM, self.num_sms, B)
            self.qkva_part = torch.zeros((s_q, B, QKVA_ROWS), device=dev, dtype=f32)
            self.o_proj_part = torch.zeros((s_o, B, HIDDEN), device=dev, dtype=f32)
            dense_k = max([lp.dense.inter for lp in self.layers if lp.dense is not None], default=0)
            s_d = split_count(HIDDEN, dense_k, self.num_sms, B) if dense_k else 1
            self.dense_part = torch.zeros((s_d, B, HIDDEN), device=dev, dtype=f32)
        self.q_abs = torch.zeros((B, N_HEADS, KV_LORA), device=dev, dtype=bf)
        self.o_lat = torch.zeros((B, N_HEADS, KV_LORA), device=dev, dtype=bf)
        self.attn_o = torch.zeros((B, N_HEADS * V_DIM), device=dev, dtype=bf)
        self.attn_out = torch.zeros((B, HIDDEN), device=dev, dtype=bf)
        self.o_part = torch.zeros((B, self.n_splits, N_HEADS, KV_LORA), device=dev, dtype=f32)
        self.ml_part = torch.zeros((B, self.n_splits, N_HEADS, 2), device=dev, dtype=f32)
        self.mla_sync = torch.zeros(B, device=dev, dtype=i32)
        # one row (small family): {first CTA, count} of the attention partials that the
        # un-absorb GEMV merges
        self.mla_parts = torch.zeros(2, device=dev, dtype=i32)
        dense = [lp.dense for lp in self.layers if lp.dense is not None]
        inter_d = max([d.inter for d in dense], default=8)
        self.mlp_h = torch.zeros((B, inter_d), device=dev, dtype=bf)
        self.mlp_out = torch.zeros((B, HIDDEN), device=dev, dtype=bf)
        moe = [lp.moe for lp in self.layers if lp.moe is not None]
        Ball = self.B_all
        if moe:
            m0 = moe[0]
            self.r_max = TOPK * Ball + 2 * B
            self.n_groups = m0.n_local + 2
            self.logits_r = torch.zeros((B, m0.n_experts), device=dev, dtype=f32)
            self.topk_ids64 = torch.zeros((B, TOPK), device=dev, dtype=i64)
            self.topk_ids32 = torch.zeros((Ball, TOPK), device=dev, dtype=i32)
            self.topk_w = torch.zeros((Ball, TOPK), device=dev, dtype=f32)
            self.ids_local = torch.zeros((B, TOPK), device=dev, dtype=i32)
            self.w_local = torch.zeros((B, TOPK), device=dev, dtype=f32)
            # per-MoE-layer group offsets (kept per layer so the routing of the last step
            # can be inspected: distinct experts per layer for the roofline)
            self.moe_index = {li: i for i, li in enumerate(l for l, lp in enumerate(self.layers)
                                                           if lp.moe is not None)}
            self.group_offsets_hist = torch.zeros((len(moe), self.n_groups + 1), device=dev, dtype=i32)
            self.route_token = torch.zeros(self.r_max, device=dev, dtype=i32)
            self.route_slot = torch.zeros(self.r_max, device=dev, dtype=i32)
            self.route_weight = torch.zeros(self.r_max, device=dev, dtype=f32)
            self.x_sorted = torch.zeros((self.r_max, HIDDEN), device=dev, dtype=bf)
            self.h_moe = torch.zeros((self.r_max, m0.inter), device=dev, dtype=bf)
            self.moe_sync = torch.zeros(self.n_groups + 2, device=dev, dtype=i32)
            # grid barrier of the single-launch router (add + RMSNorm, gate, top-6, bucketing)
            self.router_sync = torch.zeros(2, device=dev, dtype=i32)
            self.partial = torch.zeros((Ball, SLOTS, HIDDEN), device=dev, dtype=f32)
            if self.world > 1:
                self.x_all = torch.zeros((Ball, HIDDEN), device=dev, dtype=bf)
                self.moe_sum = torch.zeros((Ball, HIDDEN), device=dev, dtype=f32)
                self.moe_local = torch.zeros((B, 1, HIDDEN), device=dev, dtype=f32)
        self.logits = torch.zeros((B if self.keep_logits else 1, self.vocab), device=dev, dtype=bf)
        self.argmax_keys = torch.zeros(((self.vocab + 15) // 16) * B, device=dev, dtype=i64)
        self.step_count = torch.zeros(1, device=dev, dtype=i64)   # steps completed (peer epoch)
        self.peers = None
        if moe and self.world > 1 and self.family == ops.FAMILY_BATCH:
            self._setup_peers(len(moe))

    def _setup_peers(self, n_moe: int) -> None:
        """Expert parallel over NVLink peer memory (batch family): one buffer per rank holding
        [xg | ids | w | part | counters] (see dsv2_peer_table in include/dsv2.h), mapped by
        every rank.  The router dispatches into every rank's xg / ids / w, the fused MoE
        combines each routed slot into its owner's part; no collective runs in the step."""
        import torch.distributed as dist
        from . import _lib
        B, Ball, W = self.B, self.B_all, self.world

        def up(n):
            return (n + 255) // 256 * 256
        off_xg = 0
        off_ids = up(off_xg + Ball * HIDDEN * 2)
        off_w = up(off_ids + Ball * TOPK * 4)
        off_part = up(off_w + Ball * TOPK * 4)
        off_ctr = up(off_part + B * SLOTS * HIDDEN * 4)
        total = off_ctr + 256
        torch.cuda.synchronize(self.dev)
        local = _lib.peer_alloc(total)
        handles = [None] * W
        dist.all_gather_object(handles, _lib.peer_export(local), group=self.group)
        bases = [local if q == self.rank else _lib.peer_import(handles[q]) for q in range(W)]
        t = _lib.PeerTable()
        t.world, t.rank = W, self.rank
        for q in range(W):
            t.base[q] = bases[q]
        t.xg_offset, t.ids_offset, t.w_offset, t.part_offset, t.ctr_offset = off_xg, off_ids, off_w, off_part, off_ctr
        t.rows_per_rank, t.n_moe_layers = B, n_moe
        t.epoch = self.step_count.data_ptr()
        # time the CTAs spend in the cross-GPU waits (dispatch, combine), for the bench
        self.peer_wait_stats = torch.zeros(4, device=self.dev, dtype=torch.int64)
        t.wait_stats = self.peer_wait_stats.data_ptr()
        self.peers = t
        self._peer_local, self._peer_remote = local, [b for q, b in enumerate(bases) if q != self.rank]
        self.x_g = _device_view(local + off_xg, (Ball, HIDDEN), torch.int16, self.dev).view(torch.bfloat16)
        self.ids_g = _device_view(local + off_ids, (Ball, TOPK), torch.int32, self.dev)
        self.w_g = _device_view(local + off_w, (Ball, TOPK), torch.float32, self.dev)
        self.part_peer = _device_view(local + off_part, (B, SLOTS, HIDDEN), torch.float32, self.dev)
        dist.barrier(group=self.group)

    def close(self) -> None:
        """Unmap the other ranks' peer buffers and free this rank's (expert parallel)."""
        if self.peers is None:
            return
        from . import _lib
        torch.cuda.synchronize(self.dev)
        for b in self._peer_remote:
            _lib.peer_close(b)
        _lib.peer_free(self._peer_local)
        self.peers = None

    # ------------------------------------------------------------------ layers
    def _linear(self, **kw):
        ops.linear(family=self.family, **kw)

    def _split_linear(self, *, w, n_rows, k, x, out, **kw) -> torch.Tensor:
        """Dense linear into fp32 split-K partials out[S, B, n_rows] (batch family): every
        token stays in one tile, so the weights are streamed once, and the K split spreads
        the launch over the SMs.  Returns the [B, S, n_rows] view the consumers sum."""
        S = out.shape[0]
        self._linear(w=w, n_rows=n_rows, k=k, x=x, y=out[0], epilogue=ops.EPI_STORE_F32, n_tokens=self.B,
                     x_group_rows=self.B, k_splits=S, y_split_stride=out.stride(0), **kw)
        return out.permute(1, 0, 2)

    def _attention(self, li: int, lp: LayerPack) -> torch.Tensor:
        """Attention sublayer; returns its output (bf16 [B, 2048] or fp32 partials [B, S, 2048])."""
        a, B = lp.attn, self.B
        if self.split_k:
            self._split_linear(w=a.qkva, n_rows=QKVA_ROWS, k=HIDDEN, x=self.x, out=self.qkva_part)
            qkva = self.qkva_part
        else:
            self._linear(w=a.qkva, n_rows=QKVA_ROWS, k=HIDDEN, x=self.x, y=self.qkva, n_tokens=B,
                         x_group_rows=B)
            qkva = self.qkva
        ops.mla_prep(qkva=qkva, kv_norm_w=a.kv_norm_w, eps=a.kv_norm_eps, cos=self.cos, sin=self.sin,
                     positions=self.positions, cache=self.cache[li], q_pe_out=self.q_pe, q_nope_out=self.q_nope,
                     cache_rows=self.cache_rows)
        # q_abs[b, h] = q_nope[b, h] @ W_UK[h]
        self._linear(w=a.w_uk_t, n_rows=KV_LORA, k=QK_NOPE, w_row_stride=QK_NOPE,
                     w_group_stride=KV_LORA * QK_NOPE, x=self.q_nope, x_row_stride=N_HEADS * QK_NOPE,
                     x_group_stride=QK_NOPE, y=self.q_abs, y_row_stride=N_HEADS * KV_LORA,
                     y_group_stride=KV_LORA, n_groups=N_HEADS, n_tokens=B, w_group_rows=KV_LORA,
                     x_group_rows=B)
        defer = (self.defer_mla_merge and self.family == ops.FAMILY_SMALL and B == 1
                 and self.cache_rows is None)
        ops.mla_decode(q_abs=self.q_abs, q_pe=self.q_pe, cache=self.cache[li], positions=self.positions,
                       softmax_scale=self.scale, split_len=self.split_len, o_part=self.o_part,
                       ml_part=self.ml_part, o_lat=self.o_lat, inputs_prior=True, row_sync=self.mla_sync,
                       cache_rows=self.cache_rows, part_count=self.mla_parts if defer else None)
        # o[b, h] = o_lat[b, h] @ W_UV[h]^T,  W_UV[h] = kv_b[h*256 + 128 : h*256 + 256]
        self._linear(w=a.kv_b[QK_NOPE:], n_rows=V_DIM, k=KV_LORA, w_row_stride=KV_LORA,
                     w_group_stride=(QK_NOPE + V_DIM) * KV_LORA, x=self.o_lat, x_row_stride=N_HEADS * KV_LORA,
                     x_group_stride=KV_LORA, y=self.attn_o, y_row_stride=N_HEADS * V_DIM,
                     y_group_stride=V_DIM, n_groups=N_HEADS, n_tokens=B, w_group_rows=V_DIM,
                     x_group_rows=B, x_parts=(self.o_part, self.ml_part, self.mla_parts) if defer else None)
        if self.split_k:
            return self._split_linear(w=a.o, n_rows=HIDDEN, k=N_HEADS * V_DIM, x=self.attn_o, out=self.o_proj_part)
        self._linear(w=a.o, n_rows=HIDDEN, k=N_HEADS * V_DIM, x=self.attn_o, y=self.attn_out, n_tokens=B,
                     x_group_rows=B)
        return self.attn_out

    def _dense_mlp(self, lp: LayerPack) -> torch.Tensor:
        d, B = lp.dense, self.B
        h = self.mlp_h[:, :d.inter]
        self._linear(w=d.gate_up, n_rows=d.inter, k=HIDDEN, up_offset=d.inter * HIDDEN, x=self.x, y=h,
                     epilogue=ops.EPI_SWIGLU, n_tokens=B, w_group_rows=2 * d.inter, x_group_rows=B)
        if self.split_k:
            return self._split_linear(w=d.down, n_rows=HIDDEN, k=d.inter, x=h, out=self.dense_part)
        self._linear(w=d.down, n_rows=HIDDEN, k=d.inter, x=h, y=self.mlp_out, n_tokens=B, x_group_rows=B)
        return self.mlp_out

    def _moe(self, li: int, lp: LayerPack, attn: torch.Tensor | None = None) -> torch.Tensor:
        """MoE sublayer.  attn (one rank): the attention output still to be added to the
        residual stream; the router launch adds it and applies the post-attention RMSNorm
        itself (otherwise self.x already holds the normalised input)."""
        m, B = lp.moe, self.B
        go = self.group_offsets_hist[self.moe_index[li]]
        # batch family: the routing kernel also copies x into expert order for the TMA loads
        gather = self.x_sorted if self.family == ops.FAMILY_BATCH else None
        if self.peers is not None:
            # expert parallel over peer memory: dispatch, bucket (waits for every rank's
            # dispatch), fused MoE writing each slot into its owner's part (+ signal)
            sh, mi = self.shard, self.moe_index[li]
            ops.router(x=self.x, w=m.gate_w, scaling=m.scaling, bias=m.gate_bias, logits=self.logits_r,
                       topk_ids32=self.ids_local, topk_weights=self.w_local, topk_ids64=self.topk_ids64,
                       peers=self.peers, row_base=sh.row_lo)
            ops.moe_bucket(self.ids_g, self.w_g, m.expert_lo, m.n_local, sh.row_lo, sh.row_hi, go,
                           self.route_token, self.route_slot, self.route_weight, gather_src=self.x_g,
                           gather_out=self.x_sorted, peers=self.peers, moe_layer=mi)
            ops.moe(gate_up=m.gate_up, down=m.down, x_sorted=self.x_sorted, h=self.h_moe, group_offsets=go,
                    max_routes_per_group=self.B_all, route_slot=self.route_slot, route_weight=self.route_weight,
                    y=self.part_peer.view(-1, HIDDEN), sync=self.moe_sync, peers=self.peers)
            self._moe_pending = mi
            return self.part_peer
        if self.world == 1:
            fused = {} if attn is None else dict(residual=self.h, delta=attn, norm_w=lp.post_norm_w, eps=lp.eps)
            ops.router(x=self.x, w=m.gate_w, scaling=m.scaling, bias=m.gate_bias, logits=self.logits_r,
                       topk_ids32=self.topk_ids32, topk_weights=self.topk_w, topk_ids64=self.topk_ids64,
                       gather_out=gather, expert_lo=m.expert_lo, n_local=m.n_local, shared_lo=0,
                       shared_hi=B, group_offsets=go, route_token=self.route_token,
                       route_slot=self.route_slot, route_weight=self.route_weight, sync=self.router_sync,
                       **fused)
            x_src = self.x
        else:
            sh = self.shard
            ops.router(x=self.x, w=m.gate_w, scaling=m.scaling, bias=m.gate_bias, logits=self.logits_r,
                       topk_ids32=self.ids_local, topk_weights=self.w_local, topk_ids64=self.topk_ids64)
            gather_routing(self.x, self.ids_local, self.w_local, self.x_all, self.topk_ids32, self.topk_w,
                           group=self.group)
            ops.moe_bucket(self.topk_ids32, self.topk_w, m.expert_lo, m.n_local, sh.row_lo, sh.row_hi,
                           go, self.route_token, self.route_slot, self.route_weight,
                           gather_src=self.x_all if gather is not None else None, gather_out=gather)
            self.partial.zero_()
            x_src = self.x_all
        self._moe_gemms(m, go, x_src)
        if self.world == 1:
            return self.partial
        ops.sum_partials(self.partial, self.moe_sum)
        scatter_sum(self.moe_sum, self.moe_local.view(B, HIDDEN), group=self.group)
        return self.moe_local

    def _moe_gemms(self, m, go: torch.Tensor, x_src: torch.Tensor) -> None:
        """gate_up + SwiGLU and down + route-weight scaling over local experts + shared halves
        (batch family: one fused persistent launch; small family: two GEMV launches)."""
        if self.family == ops.FAMILY_BATCH and self.fused_moe:
            # (expert parallel: local slots only, no combine; used to time the GEMMs alone)
            ops.moe(gate_up=m.gate_up, down=m.down, x_sorted=self.x_sorted, h=self.h_moe, group_offsets=go,
                    max_routes_per_group=self.B_all, route_slot=self.route_slot,
                    route_weight=self.route_weight, y=self.partial.view(-1, HIDDEN), sync=self.moe_sync)
            return
        if self.family == ops.FAMILY_BATCH:
            gx, rx = self.x_sorted, None
        else:
            gx, rx = x_src, self.route_token
        G = self.n_groups
        self._linear(w=m.gate_up, n_rows=m.inter, k=HIDDEN, up_offset=m.inter * HIDDEN,
                     w_group_stride=2 * m.inter * HIDDEN, x=gx, y=self.h_moe, epilogue=ops.EPI_SWIGLU,
                     n_groups=G, group_offsets=go, max_routes_per_group=self.B_all,
                     route_x_row=rx, w_group_rows=2 * m.inter, x_group_rows=self.r_max, max_routes=self.r_max)
        self._linear(w=m.down, n_rows=HIDDEN, k=m.inter, w_group_stride=HIDDEN * m.inter, x=self.h_moe,
                     y=self.partial.view(-1, HIDDEN), epilogue=ops.EPI_SCALE_F32, n_groups=G,
                     group_offsets=go, max_routes_per_group=self.B_all,
                     route_y_row=self.route_slot, route_scale=self.route_weight, w_group_rows=HIDDEN,
                     x_group_rows=self.r_max, offsets_prior=True, max_routes=self.r_max)

    def time_moe_gemms(self, iters: int = 10) -> tuple[float, float, int]:
        """Replay only the grouped MoE GEMMs of every MoE layer (routing of the last step's
        last MoE layer) from a CUDA graph; returns (ms per replay, algorithmic bytes per
        replay, launches per replay).  Bytes: weights of the distinct routed experts hit plus
        the two shared-expert halves, once per layer."""
        moe_layers = [lp for lp in self.layers if lp.moe is not None]
        if not moe_layers:
            return 0.0, 0.0, 0
        go = self.group_offsets_hist[len(moe_layers) - 1]
        x_src = self.x if self.world == 1 else self.x_all
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream(device=self.dev)
        s.wait_stream(torch.cuda.current_stream(self.dev))
        from . import _lib
        n0 = _lib.kernel_launches()
        with torch.cuda.stream(s):
            for lp in moe_layers:
                self._moe_gemms(lp.moe, go, x_src)
        launches = _lib.kernel_launches() - n0
        torch.cuda.current_stream(self.dev).wait_stream(s)
        with torch.cuda.graph(g):
            for lp in moe_layers:
                self._moe_gemms(lp.moe, go, x_src)
        g.replay()
        torch.cuda.synchronize(self.dev)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(iters):
            g.replay()
        b.record()
        torch.cuda.synchronize(self.dev)
        ms = a.elapsed_time(b) / iters
        off = go.cpu()
        counts = off[1:] - off[:-1]
        m0 = moe_layers[0].moe
        per_expert = (2 * m0.inter * HIDDEN + HIDDEN * m0.inter) * 2
        nbytes = len(moe_layers) * int((counts > 0).sum()) * per_expert
        del g
        return ms, float(nbytes), launches

    # ------------------------------------------------------------------ step
    @torch.no_grad()
    def step(self, trace: dict | None = None) -> None:
        """One q_len = 1 decode step for every row (kernel launches only; graph-capturable).

        trace (eager debugging/tests only): collects the residual stream after every layer
        ("hidden", fp32 [B, 2048] each, HF output_hidden_states order starting with the
        embeddings), the router's top-6 ids of every MoE layer ("routes") and the
        normalised activations that router read ("moe_x", bf16 [B, 2048])."""
        lp0 = self.layers[0]
        ops.embed_rmsnorm(self.input_ids, self.embed, lp0.in_norm_w, lp0.eps, self.h, self.x)
        if trace is not None:
            trace.setdefault("hidden", []).append(self.h.float().clone())
            trace.setdefault("routes", [])
            trace.setdefault("moe_x", [])
        delta = None
        self._moe_pending = None
        for li, lp in enumerate(self.layers):
            if li > 0:
                self._add_rmsnorm(delta, lp.in_norm_w, lp.eps)
            attn = self._attention(li, lp)
            if lp.moe is not None and self.world == 1 and m_bf16_gate(lp):
                # one launch: residual add + RMSNorm, gate, top-6, bucketing, gather
                delta = self._moe(li, lp, attn=attn)
            else:
                ops.add_rmsnorm(self.h, attn, lp.post_norm_w, lp.eps, self.x)
                delta = self._dense_mlp(lp) if lp.dense is not None else self._moe(li, lp)
            if trace is not None:
                d = delta.float().sum(1) if delta.dim() == 3 else delta.float()
                trace["hidden"].append(self.h.float() + d)
                if lp.moe is not None:
                    trace["routes"].append(self.topk_ids64.clone())
                    trace["moe_x"].append(self.x.clone())
        self._add_rmsnorm(delta, self.final_norm_w, self.final_eps)
        if self.keep_logits:  # checking / debugging only: the greedy step needs no logits
            torch.mm(self.x, self.lm_head.t(), out=self.logits)
        # lm_head + greedy argmax in the linear's epilogue; also feeds the token back and
        # advances the positions (src/run.py:585-588)
        ops.lm_head_argmax(w=self.lm_head, x=self.x, keys=self.argmax_keys, next_ids=self.next_ids,
                           family=self.family, input_ids=self.input_ids, positions=self.positions,
                           step_counter=self.step_count)

    def _add_rmsnorm(self, delta, w, eps) -> None:
        """Residual add of the previous sublayer's output + the next RMSNorm; an expert-parallel
        MoE output first waits for every rank's combine."""
        if self._moe_pending is not None:
            ops.add_rmsnorm(self.h, delta, w, eps, self.x, peers=self.peers, moe_layer=self._moe_pending)
            self._moe_pending = None
        else:
            ops.add_rmsnorm(self.h, delta, w, eps, self.x)

    # ------------------------------------------------------------------ state
    def set_state(self, positions: torch.Tensor, input_ids: torch.Tensor) -> None:
        self.positions.copy_(positions.to(self.positions))
        self.input_ids.copy_(input_ids.to(self.input_ids).view(-1))
        self._saved = (self.positions.clone(), self.input_ids.clone())

    def restore(self) -> None:
        """Roll back positions / next tokens to the post-prefill state.  Cache rows at or
        beyond a row's position are never read before being rewritten, so the latent cache
        needs no snapshot (unlike the expanded cache of src/run.py:161-217)."""
        pos, ids = self._saved
        self.positions.copy_(pos)
        self.input_ids.copy_(ids)

    def capture(self, warmup: int = 3) -> None:
        """Warm up eagerly (rolled back), then capture one decode step in a CUDA graph."""
        s = torch.cuda.Stream(device=self.dev)
        s.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(s):
            for _ in range(warmup):
                self.step()
                self.restore()
        torch.cuda.current_stream(self.dev).wait_stream(s)
        torch.cuda.synchronize(self.dev)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self.step()
        torch.cuda.synchronize(self.dev)
        self.restore()
        self.graph = g

    def replay(self) -> None:
        self.graph.replay()

    def release(self) -> None:
        self.graph = None

    def recover(self) -> int:
        """Check the device after a step: returns the device error word (0 = every bounded
        wait and index check passed).  A nonzero word is cleared, and the progress counters
        that a launch which gave up may have left behind (the fused MoE's group counters,
        the latent attention's row tickets) are zeroed, so later steps compute correct
        results again.  Expert-parallel engines cannot recover in place (their peer
        counters follow the step count on every rank): they raise, and every rank
        rebuilds its engine."""
        from . import _lib
        torch.cuda.synchronize(self.dev)
        with torch.cuda.device(self.dev):
            code = _lib.device_error(clear=True)
            if code == 0:
                return 0
            if self.peers is not None:
                raise _lib.Dsv2Error(f"device error {code} in an expert-parallel step: rebuild the engine "
                                     "on every rank")
            s = ops.stream()
            for t in (getattr(self, "moe_sync", None), self.mla_sync):
                if t is not None:
                    _lib.reset_progress(t.data_ptr(), t.numel(), s)
            torch.cuda.synchronize(self.dev)
        return code

    # ------------------------------------------------------------------ prefill
    @torch.no_grad()
    def prefill(self, prompts: list[torch.Tensor], max_tokens_per_chunk: int = 16384,
                method: str = "kernels") -> torch.Tensor:
        """Prefill this rank's rows and return the first generated token of every row.
        method "kernels": the decode kernels run over all prompt tokens at once
        (prefill_kernels); "eager": the HF model's own forward (prefill_eager)."""
        if method == "kernels":
            return self.prefill_kernels(prompts, max_tokens_per_chunk=min(max_tokens_per_chunk, 4096))
        if method != "eager":
            raise ValueError(f"unknown prefill method {method!r}")
        return self.prefill_eager(prompts, max_tokens_per_chunk)

    @torch.no_grad()
    def prefill_kernels(self, prompts: list[torch.Tensor], max_tokens_per_chunk: int = 4096) -> torch.Tensor:
        """Prefill through the same kernels as the decode step: every prompt token is a row
        of a token batch (up to max_tokens_per_chunk tokens, across prompts); its latent
        row goes straight into this engine's cache at (sequence, position), and its
        attention reads the positions <= its own of its sequence (cache_rows), so the
        chunk's tokens attend causally in one launch.  Chunks run in prompt order, all
        layers each, so later chunks see every earlier token.  The token batch uses the
        batch (tcgen05) kernels whatever this engine's family.  Returns the greedy next
        token after each prompt (src/run.py:526-544 runs the HF forward instead)."""
        if len(prompts) != self.B:
            raise ValueError(f"expected {self.B} prompts, got {len(prompts)}")
        if not 1 <= max_tokens_per_chunk <= 4096:
            raise ValueError("max_tokens_per_chunk must be in [1, 4096] (router bucketing bound)")
        lens = [int(p.numel()) for p in prompts]
        if min(lens) < 1 or max(lens) >= self.max_len:
            raise ValueError("prompts must hold 1 .. max_len - 1 tokens")
        dev = self.dev
        tokens = torch.cat([p.view(-1).to(device=dev, dtype=torch.int64) for p in prompts])
        lens_t = torch.tensor(lens, device=dev, dtype=torch.int64)
        seq, pos, last = prefill_token_plan(lens_t)
        last = last.cpu()
        first = torch.zeros(self.B, dtype=torch.int64, device=dev)
        n = tokens.numel()
        subs: dict[int, DecodeEngine] = {}
        try:
            for c0 in range(0, n, max_tokens_per_chunk):
                c1 = min(n, c0 + max_tokens_per_chunk)
                t = c1 - c0
                sub = subs.get(t)
                if sub is None:
                    sub = DecodeEngine(self.model, t, self.max_len, "batch", cache=self.cache,
                                       gate_bias=self._gate_bias)
                    subs[t] = sub
                sub.cache_rows.copy_(seq[c0:c1])
                sub.positions.copy_(pos[c0:c1])
                sub.input_ids.copy_(tokens[c0:c1])
                sub.step()
                rows = [(b, int(last[b]) - c0) for b in range(self.B) if c0 <= int(last[b]) < c1]
                if rows:
                    bi = torch.tensor([r[0] for r in rows], device=dev)
                    ti = torch.tensor([r[1] for r in rows], device=dev)
                    first[bi] = sub.next_ids[ti]
        finally:
            for s in subs.values():
                s.close()
            subs.clear()
        self.set_state(lens_t, first)
        return first

    @torch.no_grad()
    def prefill_eager(self, prompts: list[torch.Tensor], max_tokens_per_chunk: int = 16384) -> torch.Tensor:
        """Eager HF prefill of this rank's rows (ragged prompts, right-padded in chunks).

        The latent cache rows are rebuilt from the kv_a_proj_with_mqa outputs that the HF
        forward produces: [rmsnorm(c_kv) * w | rope(k_pe)] with the same formulas as the
        decode kernel.  Returns the first generated token of every row (greedy).
        """
        if len(prompts) != self.B:
            raise ValueError(f"expected {self.B} prompts, got {len(prompts)}")
        model = self.model
        lens = [int(p.numel()) for p in prompts]
        if max(lens) >= self.max_len:
            raise ValueError("prompt longer than the cache")
        captured: dict[int, torch.Tensor] = {}
        hooks = []
        for li, layer in enumerate(model.model.layers):
            hooks.append(layer.self_attn.kv_a_proj_with_mqa.register_forward_hook(
                lambda mod, inp, out, li=li: captured.__setitem__(li, out)))
        first = torch.zeros(self.B, dtype=torch.int64, device=self.dev)
        try:
            r0 = 0
            while r0 < self.B:
                T = lens[r0]
                r1 = r0 + 1
                while r1 < self.B and (r1 - r0 + 1) * max(T, lens[r1]) <= max_tokens_per_chunk:
                    T = max(T, lens[r1])
                    r1 += 1
                nr = r1 - r0
                ids = torch.zeros((nr, T), dtype=torch.int64, device=self.dev)
                mask = torch.zeros((nr, T), dtype=torch.int64, device=self.dev)
                for i in range(nr):
                    n = lens[r0 + i]
                    ids[i, :n] = prompts[r0 + i].to(self.dev)
                    mask[i, :n] = 1
                out = model.model(input_ids=ids, attention_mask=mask, use_cache=False)
                hid = out.last_hidden_state
                idx = torch.tensor([lens[r0 + i] - 1 for i in range(nr)], device=self.dev)
                last = hid[torch.arange(nr, device=self.dev), idx]
                first[r0:r1] = torch.argmax(model.lm_head(last), dim=-1)
                for li, lp in enumerate(self.layers):
                    self.cache[li, r0:r1, :T] = latent_rows(captured[li], lp.attn.kv_norm_w,
                                                            lp.attn.kv_norm_eps, self.cos[:T], self.sin[:T])
                captured.clear()
                r0 = r1
        finally:
            for h in hooks:
                h.remove()
        pos = torch.tensor(lens, dtype=torch.int64, device=self.dev)
        self.set_state(pos, first)
        return first


def m_bf16_gate(lp: LayerPack) -> bool:
    """The MoE router of this layer runs the single-launch kernel (bf16 gate weights)."""
    return lp.moe is not None and lp.moe.gate_w.dtype == torch.bfloat16


def prefill_token_plan(lens: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Token rows of a kernel prefill: prompts of lens [B] laid end to end.  Returns the
    sequence of every token (int32, the cache row it writes and reads), its position in
    its prompt (int64) and the index of each prompt's last token (int64 [B])."""
    lens = lens.to(torch.int64)
    seq = torch.repeat_interleave(torch.arange(lens.numel(), device=lens.device, dtype=torch.int32), lens)
    starts = torch.cumsum(lens, 0) - lens
    pos = torch.arange(int(lens.sum()), device=lens.device, dtype=torch.int64) - torch.repeat_interleave(starts, lens)
    return seq, pos, torch.cumsum(lens, 0) - 1


def latent_rows(kva: torch.Tensor, norm_w: torch.Tensor, eps: float, cos: torch.Tensor,
                sin: torch.Tensor) -> torch.Tensor:
    """[.., T, 576] kv_a_proj_with_mqa output -> latent cache rows [.., T, 576] (bf16):
    bf16(c * rsqrt(mean(c^2) + eps) * w) | interleaved-pair RoPE of k_pe (fp32 math)."""
    c = kva[..., :KV_LORA].float()
    inv = torch.rsqrt(c.pow(2).mean(-1, keepdim=True) + eps)
    lat = (c * inv * norm_w.float()).to(torch.bfloat16)
    kpe = kva[..., KV_LORA:].float()
    e, o = kpe[..., 0::2], kpe[..., 1::2]
    re = e * cos - o * sin
    im = o * cos + e * sin
    rope = torch.stack([re, im], dim=-1).flatten(-2).to(torch.bfloat16)
    return torch.cat([lat, rope], dim=-1)
