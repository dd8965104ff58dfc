"""ctypes binding of libdsv2.so (the C ABI declared in include/dsv2.h).

The library is built in-tree by ``flash-deepseek-v2-lite_b200/build.py``.  There is
no fallback: if the shared object is missing or fails to load, every op raises.
Status codes map onto the exception classes the reference's wrappers raise
(``NotImplementedError`` for unsupported shape/dtype classes, ``ValueError`` for bad
arguments, ``RuntimeError`` for CUDA failures).
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libdsv2.so"

DSV2_OK = 0
DSV2_ERR_INVALID = 1
DSV2_ERR_LAUNCH = 2
DSV2_ERR_DEVICE = 3
DSV2_ERR_UNSUPPORTED = 4

DSV2_BF16 = 0
DSV2_F16 = 1
DSV2_F32 = 2

EPI_STORE_BF16 = 0
EPI_STORE_F32 = 1
EPI_SWIGLU = 2
EPI_SCALE_F32 = 3

FAMILY_SMALL = 0
FAMILY_BATCH = 1

c_i32 = ctypes.c_int32
c_i64 = ctypes.c_int64
c_f32 = ctypes.c_float
c_vp = ctypes.c_void_p


class LinearArgs(ctypes.Structure):
    _fields_ = [
        ("w", c_vp), ("w_row_stride", c_i64), ("w_group_stride", c_i64), ("up_offset", c_i64),
        ("n_rows", c_i32), ("k", c_i32),
        ("x", c_vp), ("x_row_stride", c_i64), ("x_group_stride", c_i64),
        ("y", c_vp), ("y_row_stride", c_i64), ("y_group_stride", c_i64),
        ("epilogue", c_i32), ("n_groups", c_i32), ("n_tokens", c_i32), ("max_routes_per_group", c_i32),
        ("group_offsets", c_vp), ("route_x_row", c_vp), ("route_y_row", c_vp), ("route_scale", c_vp),
        ("w_group_rows", c_i64), ("x_group_rows", c_i64),
        ("k_splits", c_i32), ("y_split_stride", c_i64), ("offsets_prior", c_i32), ("max_routes", c_i32),
        ("x_parts", c_vp), ("x_parts_ml", c_vp), ("x_parts_count", c_vp),
    ]


class PeerTable(ctypes.Structure):
    _fields_ = [
        ("world", c_i32), ("rank", c_i32), ("base", c_vp * 8),
        ("xg_offset", c_i64), ("ids_offset", c_i64), ("w_offset", c_i64), ("part_offset", c_i64),
        ("ctr_offset", c_i64), ("rows_per_rank", c_i32), ("n_moe_layers", c_i32), ("epoch", c_vp),
        ("wait_polls", c_i32), ("wait_stats", c_vp),
    ]


class MoeArgs(ctypes.Structure):
    _fields_ = [
        ("gate_up", c_vp), ("down", c_vp), ("n_groups", c_i32), ("hidden", c_i32), ("inter", c_i32),
        ("x_sorted", c_vp), ("h", c_vp), ("x_rows", c_i32), ("group_offsets", c_vp),
        ("max_routes_per_group", c_i32), ("route_slot", c_vp), ("route_weight", c_vp), ("y", c_vp),
        ("sync", c_vp), ("peers", ctypes.POINTER(PeerTable)), ("tile_tokens", c_i32),
    ]


class RouterArgs(ctypes.Structure):
    _fields_ = [
        ("x", c_vp), ("x_row_stride", c_i64), ("w", c_vp), ("w_dtype", c_i32),
        ("rows", c_i32), ("hidden", c_i32), ("n_experts", c_i32),
        ("bias", c_vp), ("scaling", c_f32),
        ("logits", c_vp), ("topk_ids64", c_vp), ("topk_ids32", c_vp), ("topk_weights", c_vp),
        ("gather_out", c_vp),
        ("expert_lo", c_i32), ("n_local", c_i32), ("shared_lo", c_i32), ("shared_hi", c_i32),
        ("group_offsets", c_vp), ("route_token", c_vp), ("route_slot", c_vp), ("route_weight", c_vp),
        ("peers", ctypes.POINTER(PeerTable)), ("row_base", c_i32),
        ("h", c_vp), ("delta", c_vp), ("delta_dtype", c_i32), ("n_delta", c_i32),
        ("delta_part_stride", c_i64), ("delta_row_stride", c_i64), ("norm_w", c_vp), ("norm_w_dtype", c_i32),
        ("eps", c_f32), ("sync", c_vp),
    ]


class MlaPrepArgs(ctypes.Structure):
    _fields_ = [
        ("qkva", c_vp), ("qkva_row_stride", c_i64), ("kv_norm_w", c_vp), ("eps", c_f32),
        ("cos_tab", c_vp), ("sin_tab", c_vp), ("rope_stride", c_i64), ("rope_rows", c_i32),
        ("positions", c_vp), ("pos_numel", c_i32),
        ("cache", c_vp), ("cache_b_stride", c_i64), ("max_len", c_i32),
        ("q_pe_out", c_vp), ("batch", c_i32),
        ("qkva_dtype", c_i32), ("qkva_parts", c_i32), ("qkva_part_stride", c_i64), ("q_nope_out", c_vp),
        ("cache_rows", c_vp), ("cache_batch", c_i32),
    ]


class MlaDecodeArgs(ctypes.Structure):
    _fields_ = [
        ("q_abs", c_vp), ("q_pe", c_vp), ("cache", c_vp), ("cache_b_stride", c_i64), ("max_len", c_i32),
        ("positions", c_vp), ("pos_numel", c_i32), ("softmax_scale", c_f32),
        ("split_len", c_i32), ("n_splits", c_i32), ("o_part", c_vp), ("ml_part", c_vp),
        ("o_lat", c_vp), ("batch", c_i32), ("inputs_prior", c_i32), ("row_sync", c_vp), ("family", c_i32),
        ("cache_rows", c_vp), ("cache_batch", c_i32), ("part_count", c_vp),
    ]


_SIGNATURES = {
    "dsv2_version": ([], c_i32),
    "dsv2_last_error": ([], ctypes.c_char_p),
    "dsv2_init": ([], c_i32),
    "dsv2_set_programmatic_launch": ([c_i32], c_i32),
    "dsv2_kernel_launches": ([], c_i64),
    "dsv2_get_device_error": ([ctypes.POINTER(c_i32), c_i32], c_i32),
    "dsv2_stream_check": ([c_vp], c_i32),
    "dsv2_reset_progress": ([c_vp, c_i64, c_vp], c_i32),
    "dsv2_rmsnorm": ([c_vp, c_i64, c_i32, c_vp, c_i32, c_vp, c_i64, c_i32, c_i32, c_f32, c_vp], c_i32),
    "dsv2_add_rmsnorm": ([c_vp, c_vp, c_vp, c_i32, c_i32, c_i64, c_i64, c_vp, c_i32, c_vp, c_i32, c_i32,
                          c_f32, ctypes.POINTER(PeerTable), c_i32, c_vp], c_i32),
    "dsv2_peer_alloc": ([ctypes.c_size_t, ctypes.POINTER(c_vp)], c_i32),
    "dsv2_peer_free": ([c_vp], c_i32),
    "dsv2_peer_export": ([c_vp, c_vp], c_i32),
    "dsv2_peer_import": ([c_vp, ctypes.POINTER(c_vp)], c_i32),
    "dsv2_peer_close": ([c_vp], c_i32),
    "dsv2_embed_rmsnorm": ([c_vp, c_vp, c_i64, c_vp, c_i32, c_vp, c_vp, c_i32, c_i32, c_f32, c_vp], c_i32),
    "dsv2_residual_add": ([c_vp, c_vp, c_vp, c_i64, c_i32, c_vp], c_i32),
    "dsv2_silu_mul": ([c_vp, c_vp, c_vp, c_i64, c_vp], c_i32),
    "dsv2_sum_partials": ([c_vp, c_i32, c_i64, c_i64, c_vp, c_i32, c_i64, c_i32, c_i32, c_vp], c_i32),
    "dsv2_prepare_decode_inputs": ([c_vp, c_i32, c_vp, c_i64, c_vp, c_i64, c_vp, c_i32, c_i32, c_vp], c_i32),
    "dsv2_copy_token_to_cache": ([c_vp, c_vp, c_vp, c_vp, c_vp, c_i32, c_i32, c_i32, c_i32, c_i32, c_i32,
                                  c_vp], c_i32),
    "dsv2_advance_positions": ([c_vp, c_i32, c_vp], c_i32),
    "dsv2_linear": ([ctypes.POINTER(LinearArgs), c_i32, c_vp], c_i32),
    "dsv2_moe": ([ctypes.POINTER(MoeArgs), c_vp], c_i32),
    "dsv2_lm_head_argmax": ([c_vp, c_i32, c_i32, c_vp, c_i64, c_i32, c_vp, c_i64, c_vp, c_vp, c_vp, c_i32, c_vp,
                             c_i32, c_vp], c_i32),
    "dsv2_router": ([ctypes.POINTER(RouterArgs), c_vp], c_i32),
    "dsv2_softmax_topk": ([c_vp, c_i32, c_i32, c_f32, c_vp, c_vp, c_vp, c_vp], c_i32),
    "dsv2_moe_bucket": ([c_vp, c_vp, c_i32, c_i32, c_i32, c_i32, c_i32, c_vp, c_vp, c_vp, c_vp,
                         c_vp, c_i64, c_vp, c_i32, ctypes.POINTER(PeerTable), c_i32, c_vp], c_i32),
    "dsv2_gather_rows": ([c_vp, c_i64, c_vp, c_vp, c_i32, c_vp, c_i32, c_i32, c_vp], c_i32),
    "dsv2_mla_prep": ([ctypes.POINTER(MlaPrepArgs), c_vp], c_i32),
    "dsv2_mla_decode": ([ctypes.POINTER(MlaDecodeArgs), c_vp], c_i32),
    "dsv2_mla_decode_noalloc": ([c_vp, c_vp, c_vp, c_i64, c_i32, c_vp, c_i32, c_f32, c_i32, c_vp, c_i32, c_vp],
                                c_i32),
}

EXPORTED = tuple(_SIGNATURES)

_lib = None


class Dsv2Error(RuntimeError):
    """CUDA launch/driver failure or a device-side error reported by libdsv2."""


def load(path: str | os.PathLike | None = None) -> ctypes.CDLL:
    """Load libdsv2.so once and declare every entry point's signature."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path is not None else LIB_PATH
    if not p.exists():
        raise ImportError(
            f"libdsv2.so not found at {p}; build it with `python flash-deepseek-v2-lite_b200/build.py`")
    lib = ctypes.CDLL(str(p))
    for name, (argtypes, restype) in _SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = argtypes
        fn.restype = restype
    if path is None:
        _lib = lib
    return lib


def check(rc: int, what: str) -> None:
    if rc == DSV2_OK:
        return
    msg = load().dsv2_last_error().decode(errors="replace")
    text = f"{what}: {msg}" if msg else what
    if rc == DSV2_ERR_INVALID:
        raise ValueError(text)
    if rc == DSV2_ERR_UNSUPPORTED:
        raise NotImplementedError(text)
    raise Dsv2Error(text)


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args), name)


def peer_alloc(nbytes: int) -> int:
    """cudaMalloc'd, zeroed device buffer that other processes can map (expert parallel)."""
    ptr = c_vp()
    check(load().dsv2_peer_alloc(nbytes, ctypes.byref(ptr)), "dsv2_peer_alloc")
    return int(ptr.value)


def peer_export(ptr: int) -> bytes:
    handle = ctypes.create_string_buffer(64)
    check(load().dsv2_peer_export(ptr, handle), "dsv2_peer_export")
    return handle.raw


def peer_import(handle: bytes) -> int:
    ptr = c_vp()
    buf = ctypes.create_string_buffer(handle, 64)
    check(load().dsv2_peer_import(buf, ctypes.byref(ptr)), "dsv2_peer_import")
    return int(ptr.value)


def peer_close(ptr: int) -> None:
    check(load().dsv2_peer_close(ptr), "dsv2_peer_close")


def peer_free(ptr: int) -> None:
    check(load().dsv2_peer_free(ptr), "dsv2_peer_free")


def kernel_launches() -> int:
    """Kernels enqueued by libdsv2 so far in this process."""
    return int(load().dsv2_kernel_launches())


def set_programmatic_launch(enable: bool) -> bool:
    """Turn programmatic dependent launch on or off for later launches; returns the old setting."""
    return bool(load().dsv2_set_programmatic_launch(1 if enable else 0))


def device_error(clear: bool = True) -> int:
    """Synchronously read (and clear) the device error word of the current device."""
    code = c_i32(0)
    check(load().dsv2_get_device_error(ctypes.byref(code), 1 if clear else 0), "dsv2_get_device_error")
    return int(code.value)


def stream_check(stream: int | None) -> None:
    """Wait for `stream` and raise Dsv2Error if the device error word is set (not cleared)."""
    check(load().dsv2_stream_check(stream), "dsv2_stream_check")


def reset_progress(counters, count: int, stream: int | None) -> None:
    """Zero `count` int32 progress counters (MoE group counters, attention row tickets) on `stream`."""
    check(load().dsv2_reset_progress(counters, count, stream), "dsv2_reset_progress")
