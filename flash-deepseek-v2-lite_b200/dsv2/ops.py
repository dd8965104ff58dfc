"""Tensor-level wrappers over the libdsv2 C ABI.

Every function enqueues on the current torch CUDA stream, writes into caller-owned
output tensors and never synchronises, so the whole decode step can be captured in
a CUDA graph.  Validation mirrors the reference wrappers' checks (device, dtype,
contiguity) and raises the same exception classes.
"""
from __future__ import annotations

import ctypes
import math

import torch

from . import _lib
from ._lib import (
    DSV2_BF16, DSV2_F16, DSV2_F32, EPI_STORE_BF16, EPI_STORE_F32, EPI_SWIGLU, EPI_SCALE_F32,
    FAMILY_SMALL, FAMILY_BATCH, LinearArgs, MlaDecodeArgs, MlaPrepArgs, MoeArgs, PeerTable, RouterArgs,
)

__all__ = [
    "stream", "rmsnorm", "add_rmsnorm", "embed_rmsnorm", "residual_add", "silu_mul", "sum_partials",
    "prepare_decode_inputs", "copy_token_to_cache", "advance_positions", "linear",
    "router", "softmax_topk", "moe_bucket", "gather_rows", "moe", "mla_prep", "mla_decode", "mla_splits", "mla_workspace", "lm_head_argmax",
    "EPI_STORE_BF16", "EPI_STORE_F32", "EPI_SWIGLU", "EPI_SCALE_F32", "FAMILY_SMALL", "FAMILY_BATCH",
]


def stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _cuda(t: torch.Tensor, name: str) -> None:
    if t.device.type != "cuda":
        raise NotImplementedError(f"{name} must be a CUDA tensor")


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _wdtype(w: torch.Tensor) -> int:
    if w.dtype == torch.bfloat16:
        return DSV2_BF16
    if w.dtype == torch.float32:
        return DSV2_F32
    if w.dtype == torch.float16:
        return DSV2_F16
    raise NotImplementedError(f"unsupported weight dtype {w.dtype}")


_ACT16 = {torch.bfloat16: DSV2_BF16, torch.float16: DSV2_F16}


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float, out: torch.Tensor) -> torch.Tensor:
    """out[r] = x[r] * rsqrt(mean(x[r]^2) + eps) * w for 2-D x (rows, cols), fp32 math, one
    rounding to x's dtype (bf16 or fp16)."""
    _cuda(x, "x")
    if x.dtype not in _ACT16 or out.dtype != x.dtype:
        raise NotImplementedError("rmsnorm supports bf16 / fp16 activations (out in the same dtype)")
    if x.stride(-1) != 1 or out.stride(-1) != 1 or not w.is_contiguous():
        raise NotImplementedError("rmsnorm requires a contiguous last dimension and weight")
    rows, cols = x.shape
    _lib.call("dsv2_rmsnorm", x.data_ptr(), x.stride(0), _ACT16[x.dtype], w.data_ptr(), _wdtype(w),
              out.data_ptr(), out.stride(0), rows, cols, float(eps), stream())
    return out


def _peers_ref(peers: PeerTable | None):
    return None if peers is None else ctypes.byref(peers)


def add_rmsnorm(h: torch.Tensor, delta: torch.Tensor | None, w: torch.Tensor | None, eps: float,
                y: torch.Tensor | None, h_out: torch.Tensor | None = None, peers: PeerTable | None = None,
                moe_layer: int = 0) -> None:
    """h(_out) = bf16(h + sum of delta parts); y = rmsnorm(h(_out)) * w.

    delta: None, bf16 [rows, cols], or fp32 [rows, parts, cols] (summed over parts).
    peers / moe_layer: delta is the expert-parallel part buffer of MoE layer moe_layer
    (waits for every rank's combine first).
    """
    _cuda(h, "h")
    rows, cols = h.shape
    if delta is None:
        dptr, ddt, nd, dps, drs = None, DSV2_BF16, 0, 0, 0
    elif delta.dim() == 2:
        if delta.dtype != torch.bfloat16:
            raise NotImplementedError("2-D delta must be bf16")
        dptr, ddt, nd, dps, drs = delta.data_ptr(), DSV2_BF16, 1, 0, delta.stride(0)
    else:
        if delta.dtype != torch.float32:
            raise NotImplementedError("3-D delta (per-slot partials) must be fp32")
        dptr, ddt, nd, dps, drs = delta.data_ptr(), DSV2_F32, delta.shape[1], delta.stride(1), delta.stride(0)
    _lib.call("dsv2_add_rmsnorm", h.data_ptr(), _ptr(h_out), dptr, ddt, nd, dps, drs,
              _ptr(w), _wdtype(w) if w is not None else DSV2_BF16, _ptr(y), rows, cols, float(eps),
              _peers_ref(peers), moe_layer, stream())


def embed_rmsnorm(ids: torch.Tensor, table: torch.Tensor, w: torch.Tensor, eps: float,
                  h: torch.Tensor, y: torch.Tensor) -> None:
    if ids.dtype != torch.int64:
        raise ValueError("ids must be int64")
    rows, cols = h.shape
    _lib.call("dsv2_embed_rmsnorm", ids.data_ptr(), table.data_ptr(), table.shape[0], w.data_ptr(),
              _wdtype(w), h.data_ptr(), y.data_ptr(), rows, cols, float(eps), stream())


def residual_add(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    """out = a + b in fp32, rounded once to the inputs' dtype (bf16 or fp16)."""
    if a.dtype not in _ACT16 or b.dtype != a.dtype or out.dtype != a.dtype:
        raise NotImplementedError("residual_add supports bf16 / fp16 tensors of one dtype")
    _lib.call("dsv2_residual_add", a.data_ptr(), b.data_ptr(), out.data_ptr(), a.numel(), _ACT16[a.dtype],
              stream())
    return out


def silu_mul(gate: torch.Tensor, up: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    _lib.call("dsv2_silu_mul", gate.data_ptr(), up.data_ptr(), out.data_ptr(), gate.numel(), stream())
    return out


def sum_partials(part: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    """out[r] = sum_p part[r, p] (fp32 partials [rows, parts, cols], summed in part order)
    stored as out's dtype (bf16 or fp32)."""
    _cuda(part, "part")
    if part.dtype != torch.float32 or part.dim() != 3 or part.stride(2) != 1:
        raise NotImplementedError("sum_partials expects fp32 partials [rows, parts, cols] with contiguous cols")
    rows, parts, cols = part.shape
    if tuple(out.shape) != (rows, cols) or out.stride(1) != 1:
        raise ValueError("out must be [rows, cols] with contiguous cols")
    if out.dtype == torch.bfloat16:
        odt = DSV2_BF16
    elif out.dtype == torch.float32:
        odt = DSV2_F32
    else:
        raise NotImplementedError(f"sum_partials output dtype {out.dtype}")
    _lib.call("dsv2_sum_partials", part.data_ptr(), parts, part.stride(1), part.stride(0), out.data_ptr(), odt,
              out.stride(0), rows, cols, stream())
    return out


def prepare_decode_inputs(cache_position: torch.Tensor, attention_mask: torch.Tensor | None,
                          position_ids: torch.Tensor | None, attention_mask_index: torch.Tensor | None,
                          batch: int, max_len: int) -> None:
    _lib.call("dsv2_prepare_decode_inputs", cache_position.data_ptr(), cache_position.numel(),
              _ptr(attention_mask), attention_mask.stride(0) if attention_mask is not None else 0,
              _ptr(position_ids), position_ids.stride(0) if position_ids is not None else 0,
              _ptr(attention_mask_index), batch, max_len, stream())


def copy_token_to_cache(src: torch.Tensor, dst: torch.Tensor, cache_position: torch.Tensor) -> None:
    """dst[b, h, pos_b, :] = src[b, h, 0, :]  (src [B, H, 1, D], dst [B, H, S, D])."""
    ss = (ctypes.c_int64 * 3)(src.stride(0), src.stride(1), src.stride(3))
    ds = (ctypes.c_int64 * 4)(*dst.stride())
    _lib.call("dsv2_copy_token_to_cache", src.data_ptr(), ss, dst.data_ptr(), ds, cache_position.data_ptr(),
              cache_position.numel(), src.shape[0], src.shape[1], src.shape[3], src.element_size(),
              dst.shape[2], stream())


def advance_positions(pos: torch.Tensor) -> None:
    _lib.call("dsv2_advance_positions", pos.data_ptr(), pos.numel(), stream())


def linear(*, w: torch.Tensor, n_rows: int, k: int, x: torch.Tensor | None, y: torch.Tensor,
           family: int, epilogue: int = EPI_STORE_BF16,
           w_row_stride: int | None = None, w_group_stride: int = 0, up_offset: int = 0,
           x_row_stride: int | None = None, x_group_stride: int = 0,
           y_row_stride: int | None = None, y_group_stride: int = 0,
           n_groups: int = 1, n_tokens: int = 0,
           group_offsets: torch.Tensor | None = None, max_routes_per_group: int = 0,
           route_x_row: torch.Tensor | None = None, route_y_row: torch.Tensor | None = None,
           route_scale: torch.Tensor | None = None,
           w_group_rows: int | None = None, x_group_rows: int | None = None,
           x_base: int | None = None, k_splits: int = 1, y_split_stride: int = 0,
           offsets_prior: bool = False, max_routes: int = 0,
           x_parts: tuple | None = None) -> None:
    """Generic linear (see dsv2_linear_args in include/dsv2.h).

    x_parts (small family, one token): (o_part, ml_part, part_count) of a mla_decode call
    that left its partials unmerged; the activation rows are merged from them (x unused).

    Strides are in elements; defaults take them from the 2-D views of w / x / y.
    x_base overrides x's data pointer (strided column views such as q_nope).
    offsets_prior: group_offsets / route arrays were written at least two launches earlier
    on this stream (lets the kernel start before the previous one completes).
    """
    a = LinearArgs()
    a.w = w.data_ptr()
    a.w_row_stride = w.stride(-2) if w_row_stride is None else w_row_stride
    a.w_group_stride = w_group_stride
    a.up_offset = up_offset
    a.n_rows = n_rows
    a.k = k
    if x is None and x_parts is None:
        raise ValueError("linear: x or x_parts is required")
    a.x = (x.data_ptr() if x is not None else None) if x_base is None else x_base
    a.x_row_stride = (x.stride(-2) if x is not None else k) if x_row_stride is None else x_row_stride
    a.x_group_stride = x_group_stride
    a.y = y.data_ptr()
    a.y_row_stride = y.stride(-2) if y_row_stride is None else y_row_stride
    a.y_group_stride = y_group_stride
    a.epilogue = epilogue
    a.n_groups = n_groups
    a.n_tokens = n_tokens
    a.max_routes_per_group = max_routes_per_group
    a.group_offsets = _ptr(group_offsets)
    a.route_x_row = _ptr(route_x_row)
    a.route_y_row = _ptr(route_y_row)
    a.route_scale = _ptr(route_scale)
    a.w_group_rows = n_rows if w_group_rows is None else w_group_rows
    a.x_group_rows = (n_tokens if x_group_rows is None else x_group_rows)
    a.k_splits = k_splits
    a.y_split_stride = y_split_stride
    a.offsets_prior = 1 if offsets_prior else 0
    a.max_routes = max_routes
    if x_parts is not None:
        o_part, ml_part, part_count = x_parts
        for name, t in (("o_part", o_part), ("ml_part", ml_part), ("part_count", part_count)):
            _cuda(t, name)
        if o_part.dtype != torch.float32 or ml_part.dtype != torch.float32 or part_count.dtype != torch.int32:
            raise ValueError("linear: x_parts are (fp32 o_part, fp32 ml_part, int32 part_count)")
        a.x_parts, a.x_parts_ml, a.x_parts_count = o_part.data_ptr(), ml_part.data_ptr(), part_count.data_ptr()
    _lib.call("dsv2_linear", ctypes.byref(a), family, stream())


def moe(*, gate_up: torch.Tensor, down: torch.Tensor, x_sorted: torch.Tensor, h: torch.Tensor,
        group_offsets: torch.Tensor, max_routes_per_group: int, route_slot: torch.Tensor,
        route_weight: torch.Tensor, y: torch.Tensor, sync: torch.Tensor, tile_tokens: int = 0,
        peers: PeerTable | None = None) -> None:
    """Fused grouped MoE of one layer (batch family): gate_up + SwiGLU -> h, then down scaled
    by the route weight into y[route_slot] (fp32 rows).  See dsv2_moe_args in include/dsv2.h.
    gate_up [G, 2I, H], down [G, H, I] bf16; x_sorted [R, H], h [R, I] bf16; sync int32 [G + 2]
    (zero-initialised once, left zero by every call)."""
    for name, t in (("gate_up", gate_up), ("down", down), ("x_sorted", x_sorted), ("h", h), ("y", y)):
        _cuda(t, name)
        if not t.is_contiguous():
            raise NotImplementedError(f"moe requires a contiguous {name}")
    if gate_up.dtype != torch.bfloat16 or down.dtype != torch.bfloat16 or x_sorted.dtype != torch.bfloat16:
        raise NotImplementedError("moe supports bf16 weights and activations")
    if y.dtype != torch.float32 or sync.dtype != torch.int32 or group_offsets.dtype != torch.int32:
        raise NotImplementedError("moe: y must be fp32, sync and group_offsets int32")
    G, two_i, H = gate_up.shape
    inter = two_i // 2
    if tuple(down.shape) != (G, H, inter) or x_sorted.shape[1] != H or tuple(h.shape) != (x_sorted.shape[0], inter):
        raise ValueError("moe: inconsistent shapes")
    if sync.numel() < G + 2 or group_offsets.numel() < G + 1:
        raise ValueError("moe: sync needs n_groups + 2 entries and group_offsets n_groups + 1")
    a = MoeArgs()
    a.gate_up, a.down = gate_up.data_ptr(), down.data_ptr()
    a.n_groups, a.hidden, a.inter = G, H, inter
    a.x_sorted, a.h, a.x_rows = x_sorted.data_ptr(), h.data_ptr(), x_sorted.shape[0]
    a.group_offsets = group_offsets.data_ptr()
    a.max_routes_per_group = max_routes_per_group
    a.route_slot, a.route_weight = route_slot.data_ptr(), route_weight.data_ptr()
    a.y, a.sync = y.data_ptr(), sync.data_ptr()
    a.tile_tokens = tile_tokens
    if peers is not None:
        a.peers = ctypes.pointer(peers)
    _lib.call("dsv2_moe", ctypes.byref(a), stream())


def lm_head_argmax(*, w: torch.Tensor, x: torch.Tensor, keys: torch.Tensor, next_ids: torch.Tensor,
                   family: int, input_ids: torch.Tensor | None = None,
                   positions: torch.Tensor | None = None, step_counter: torch.Tensor | None = None) -> None:
    """next_ids[t] = argmax over the vocabulary of bf16(x[t] @ w^T) (lowest index on ties),
    without materialising the logits; optionally input_ids = next_ids and positions += 1.
    keys: uint64 (int64) work buffer of at least ceil(vocab / 16) * tokens entries."""
    _cuda(x, "x")
    if w.dtype != torch.bfloat16 or x.dtype != torch.bfloat16 or w.stride(1) != 1 or x.stride(1) != 1:
        raise NotImplementedError("lm_head_argmax supports bf16 weights/activations with contiguous rows")
    if next_ids.dtype != torch.int64 or keys.dtype not in (torch.int64, torch.uint64):
        raise ValueError("next_ids must be int64 and keys 64-bit")
    vocab, hidden = w.shape
    n = x.shape[0]
    _lib.call("dsv2_lm_head_argmax", w.data_ptr(), vocab, hidden, x.data_ptr(), x.stride(0), n, keys.data_ptr(),
              keys.numel(), next_ids.data_ptr(), _ptr(input_ids), _ptr(positions),
              positions.numel() if positions is not None else 0, _ptr(step_counter), family, stream())


def router(*, x: torch.Tensor, w: torch.Tensor, scaling: float, logits: torch.Tensor,
           topk_ids32: torch.Tensor, topk_weights: torch.Tensor, topk_ids64: torch.Tensor | None = None,
           bias: torch.Tensor | None = None, gather_out: torch.Tensor | None = None,
           expert_lo: int = 0, n_local: int = 0, shared_lo: int = 0, shared_hi: int = 0,
           group_offsets: torch.Tensor | None = None, route_token: torch.Tensor | None = None,
           route_slot: torch.Tensor | None = None, route_weight: torch.Tensor | None = None,
           peers: PeerTable | None = None, row_base: int = 0, residual: torch.Tensor | None = None,
           delta: torch.Tensor | None = None, norm_w: torch.Tensor | None = None, eps: float = 0.0,
           sync: torch.Tensor | None = None) -> None:
    """Gate logits + softmax + top-6 (+ bucketing when group_offsets is given, + the
    expert-ordered copy of x into gather_out when given; + expert-parallel dispatch of
    x / ids / weights to every rank's peer buffer when peers is given).

    residual / delta / norm_w / eps (bf16 gate, one rank): the router's input is formed in
    the same launch, residual = bf16(residual + delta) in place and x = rmsnorm(residual) *
    norm_w written into x (delta: bf16 [rows, cols] or fp32 partials [rows, parts, cols],
    as add_rmsnorm).  sync (int32 [2], zeroed once): the bucketing runs in the same launch."""
    a = RouterArgs()
    a.x = x.data_ptr()
    a.x_row_stride = x.stride(0)
    a.w = w.data_ptr()
    a.w_dtype = _wdtype(w)
    a.rows = x.shape[0]
    a.hidden = x.shape[1]
    a.n_experts = w.shape[0]
    a.bias = _ptr(bias)
    a.scaling = float(scaling)
    a.logits = logits.data_ptr()
    a.topk_ids64 = _ptr(topk_ids64)
    a.topk_ids32 = topk_ids32.data_ptr()
    a.topk_weights = topk_weights.data_ptr()
    a.gather_out = _ptr(gather_out)
    a.expert_lo, a.n_local, a.shared_lo, a.shared_hi = expert_lo, n_local, shared_lo, shared_hi
    a.group_offsets = _ptr(group_offsets)
    a.route_token = _ptr(route_token)
    a.route_slot = _ptr(route_slot)
    a.route_weight = _ptr(route_weight)
    if peers is not None:
        a.peers = ctypes.pointer(peers)
    a.row_base = row_base
    if residual is not None:
        _cuda(residual, "residual")
        if residual.dtype != torch.bfloat16 or not residual.is_contiguous() or residual.shape != x.shape:
            raise NotImplementedError("residual must be a contiguous bf16 tensor shaped like x")
        a.h = residual.data_ptr()
        a.norm_w = norm_w.data_ptr()
        a.norm_w_dtype = _wdtype(norm_w)
        a.eps = float(eps)
        if delta is not None:
            if delta.dim() == 2:
                if delta.dtype != torch.bfloat16:
                    raise NotImplementedError("2-D delta must be bf16")
                a.delta, a.delta_dtype, a.n_delta = delta.data_ptr(), DSV2_BF16, 1
                a.delta_part_stride, a.delta_row_stride = 0, delta.stride(0)
            else:
                if delta.dtype != torch.float32:
                    raise NotImplementedError("3-D delta (per-part partials) must be fp32")
                a.delta, a.delta_dtype, a.n_delta = delta.data_ptr(), DSV2_F32, delta.shape[1]
                a.delta_part_stride, a.delta_row_stride = delta.stride(1), delta.stride(0)
    if sync is not None:
        if sync.dtype != torch.int32 or sync.numel() < 2:
            raise ValueError("sync must be int32 with 2 entries")
        a.sync = sync.data_ptr()
    _lib.call("dsv2_router", ctypes.byref(a), stream())


def softmax_topk(logits: torch.Tensor, scaling: float, topk_ids64: torch.Tensor | None,
                 topk_ids32: torch.Tensor, topk_weights: torch.Tensor) -> None:
    _lib.call("dsv2_softmax_topk", logits.data_ptr(), logits.shape[0], logits.shape[1], float(scaling),
              _ptr(topk_ids64), topk_ids32.data_ptr(), topk_weights.data_ptr(), stream())


def moe_bucket(topk_ids32: torch.Tensor, topk_weights: torch.Tensor, expert_lo: int, n_local: int,
               shared_lo: int, shared_hi: int, group_offsets: torch.Tensor, route_token: torch.Tensor,
               route_slot: torch.Tensor, route_weight: torch.Tensor, gather_src: torch.Tensor | None = None,
               gather_out: torch.Tensor | None = None, peers: PeerTable | None = None,
               moe_layer: int = 0) -> None:
    _lib.call("dsv2_moe_bucket", topk_ids32.data_ptr(), topk_weights.data_ptr(), topk_ids32.shape[0],
              expert_lo, n_local, shared_lo, shared_hi, group_offsets.data_ptr(), route_token.data_ptr(),
              route_slot.data_ptr(), route_weight.data_ptr(), _ptr(gather_src),
              gather_src.stride(0) if gather_src is not None else 0, _ptr(gather_out),
              gather_src.shape[1] if gather_src is not None else 0, _peers_ref(peers), moe_layer, stream())


def gather_rows(x: torch.Tensor, route_token: torch.Tensor, group_offsets: torch.Tensor,
                n_groups: int, out: torch.Tensor, max_routes: int) -> None:
    _lib.call("dsv2_gather_rows", x.data_ptr(), x.stride(0), route_token.data_ptr(),
              group_offsets.data_ptr(), n_groups, out.data_ptr(), x.shape[1], max_routes, stream())


def _check_cache(cache: torch.Tensor) -> None:
    _cuda(cache, "cache")
    if cache.dim() != 3 or cache.shape[2] != 576 or cache.stride(2) != 1 or cache.stride(1) != 576:
        raise NotImplementedError("latent cache must be [B, max_len, 576] with contiguous 576-wide rows")


def mla_prep(*, qkva: torch.Tensor, kv_norm_w: torch.Tensor, eps: float, cos: torch.Tensor,
             sin: torch.Tensor, positions: torch.Tensor, cache: torch.Tensor,
             q_pe_out: torch.Tensor, q_nope_out: torch.Tensor | None = None,
             cache_rows: torch.Tensor | None = None) -> None:
    """New-token preparation for one layer.

    qkva: bf16 [B, 3648], or fp32 split-K partial sums [S, B, 3648] (summed here);
    cache: [rows, max_len, 576] (one layer); positions int64 [1] or [B];
    q_nope_out (optional): bf16 [B, 16, 128] copy of the (summed) q_nope;
    cache_rows (optional): int32 [B], the cache row of each input row (default: row b)."""
    _cuda(qkva, "qkva")
    if qkva.dim() == 2 and qkva.dtype == torch.bfloat16:
        dt, parts, pstride, rstride, batch = DSV2_BF16, 1, 0, qkva.stride(0), qkva.shape[0]
    elif qkva.dim() == 3 and qkva.dtype == torch.float32:
        dt, parts, pstride, rstride, batch = DSV2_F32, qkva.shape[0], qkva.stride(0), qkva.stride(1), qkva.shape[1]
    else:
        raise NotImplementedError("mla_prep expects bf16 qkva [B, 3648] or fp32 partials [S, B, 3648]")
    if qkva.stride(-1) != 1 or qkva.shape[-1] != 3648:
        raise NotImplementedError("mla_prep expects 3648-wide rows with a contiguous last dimension")
    if not q_pe_out.is_contiguous() or cos.stride(1) != 1 or sin.stride(1) != 1:
        raise NotImplementedError("mla_prep requires contiguous q_pe_out and rope tables")
    if q_nope_out is not None and (not q_nope_out.is_contiguous() or q_nope_out.dtype != torch.bfloat16):
        raise NotImplementedError("q_nope_out must be a contiguous bf16 [B, 16, 128] tensor")
    if cos.dtype != torch.float32 or sin.dtype != torch.float32:
        raise NotImplementedError("rope tables must be fp32")
    _check_cache(cache)
    a = MlaPrepArgs()
    a.qkva = qkva.data_ptr()
    a.qkva_row_stride = rstride
    a.kv_norm_w = kv_norm_w.data_ptr()
    a.eps = float(eps)
    a.cos_tab = cos.data_ptr()
    a.sin_tab = sin.data_ptr()
    a.rope_stride = cos.stride(0)
    a.rope_rows = cos.shape[0]
    a.positions = positions.data_ptr()
    a.pos_numel = positions.numel()
    a.cache = cache.data_ptr()
    a.cache_b_stride = cache.stride(0)
    a.max_len = cache.shape[1]
    a.q_pe_out = q_pe_out.data_ptr()
    a.batch = batch
    a.qkva_dtype = dt
    a.qkva_parts = parts
    a.qkva_part_stride = pstride
    a.q_nope_out = _ptr(q_nope_out)
    a.cache_batch = cache.shape[0]
    if cache_rows is not None:
        _cuda(cache_rows, "cache_rows")
        if cache_rows.dtype != torch.int32 or cache_rows.numel() < batch:
            raise ValueError("cache_rows must be int32 with one entry per input row")
        a.cache_rows = cache_rows.data_ptr()
    elif cache.shape[0] < batch:
        raise ValueError("the cache has fewer rows than the batch (pass cache_rows)")
    _lib.call("dsv2_mla_prep", ctypes.byref(a), stream())


MLA_MAX_CTAS = 160   # CTAs of the balanced latent-attention kernel (at most one per SM)


def mla_splits(batch: int, max_len: int, split_len: int, num_sms: int, family: int = FAMILY_SMALL) -> int:
    """n_splits of the [B, n_splits, 16, 512] / [B, n_splits, 16, 2] partial buffers:
    FAMILY_SMALL (balanced kernel) needs two slots per CTA, FAMILY_BATCH (split grid) one
    per split of the longest row."""
    if family == FAMILY_SMALL:
        return max(1, math.ceil(2 * min(num_sms, MLA_MAX_CTAS) / batch))
    return math.ceil(max_len / split_len)


def mla_workspace(batch: int, max_len: int, split_len: int, device, family: int = FAMILY_SMALL) -> dict:
    """Work buffers of mla_decode: o_part, ml_part and (FAMILY_SMALL) the zeroed row tickets."""
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    n = mla_splits(batch, max_len, split_len, sms, family)
    ws = {"o_part": torch.zeros((batch, n, 16, 512), device=device, dtype=torch.float32),
          "ml_part": torch.zeros((batch, n, 16, 2), device=device, dtype=torch.float32)}
    if family == FAMILY_SMALL:
        ws["row_sync"] = torch.zeros(batch, device=device, dtype=torch.int32)
    return ws


def mla_decode(*, q_abs: torch.Tensor, q_pe: torch.Tensor, cache: torch.Tensor, positions: torch.Tensor,
               softmax_scale: float, split_len: int, o_part: torch.Tensor, ml_part: torch.Tensor,
               o_lat: torch.Tensor, inputs_prior: bool = False, row_sync: torch.Tensor | None = None,
               family: int = FAMILY_SMALL, cache_rows: torch.Tensor | None = None,
               part_count: torch.Tensor | None = None) -> None:
    """Latent attention for every row (see dsv2_mla_decode_args in include/dsv2.h).
    part_count (FAMILY_SMALL, one row, optional int32 [2]): leave the partials unmerged for
    a following linear(x_parts=...); o_lat is then not written.
    inputs_prior: q_pe, positions and the cache were written at least two launches earlier
    on this stream (only q_abs by the previous one).
    family FAMILY_SMALL: balanced mma.sync kernel, one launch; split_len = fewest positions
    per CTA (multiple of 32); row_sync (int32 [B], zero-initialised, left zero) required.
    family FAMILY_BATCH: tcgen05 kernel over split_len-position splits + merge launch.
    cache_rows (FAMILY_SMALL, optional): int32 [B], the cache row each query row reads
    (kernel prefill: the tokens of one sequence attend causally through their positions).
    Buffers: see mla_workspace."""
    for name, t in (("q_abs", q_abs), ("q_pe", q_pe), ("o_part", o_part), ("ml_part", ml_part), ("o_lat", o_lat)):
        _cuda(t, name)
        if not t.is_contiguous():
            raise NotImplementedError(f"mla_decode requires a contiguous {name}")
    if q_abs.dtype != torch.bfloat16 or q_pe.dtype != torch.bfloat16 or cache.dtype != torch.bfloat16:
        raise NotImplementedError("mla_decode supports bf16 queries and cache only")
    if tuple(q_abs.shape[1:]) != (16, 512) or tuple(q_pe.shape[1:]) != (16, 64):
        raise ValueError("q_abs must be [B, 16, 512] and q_pe [B, 16, 64]")
    _check_cache(cache)
    a = MlaDecodeArgs()
    a.q_abs = q_abs.data_ptr()
    a.q_pe = q_pe.data_ptr()
    a.cache = cache.data_ptr()
    a.cache_b_stride = cache.stride(0)
    a.max_len = cache.shape[1]
    a.positions = positions.data_ptr()
    a.pos_numel = positions.numel()
    a.softmax_scale = float(softmax_scale)
    a.split_len = split_len
    a.n_splits = o_part.shape[1]
    a.o_part = o_part.data_ptr()
    a.ml_part = ml_part.data_ptr()
    a.o_lat = o_lat.data_ptr()
    a.batch = q_abs.shape[0]
    a.inputs_prior = 1 if inputs_prior else 0
    a.family = family
    a.cache_batch = cache.shape[0]
    if cache_rows is not None:
        _cuda(cache_rows, "cache_rows")
        if cache_rows.dtype != torch.int32 or cache_rows.numel() < q_abs.shape[0]:
            raise ValueError("cache_rows must be int32 with one entry per query row")
        a.cache_rows = cache_rows.data_ptr()
    elif cache.shape[0] < q_abs.shape[0]:
        raise ValueError("the cache has fewer rows than the batch (pass cache_rows)")
    if family == FAMILY_SMALL and row_sync is None:
        raise ValueError("mla_decode: row_sync (int32 [B], zeroed) is required; see mla_workspace")
    if row_sync is not None:
        _cuda(row_sync, "row_sync")
        if row_sync.dtype != torch.int32 or row_sync.numel() < q_abs.shape[0]:
            raise ValueError("row_sync must be int32 with one entry per row")
        a.row_sync = row_sync.data_ptr()
    if part_count is not None:
        _cuda(part_count, "part_count")
        if part_count.dtype != torch.int32 or part_count.numel() < 2:
            raise ValueError("part_count must be int32 [2]")
        a.part_count = part_count.data_ptr()
    _lib.call("dsv2_mla_decode", ctypes.byref(a), stream())
