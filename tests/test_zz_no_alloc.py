"""The allocation-free latent-attention entry point (dsv2_mla_decode_noalloc).

Some callers of this library cannot allocate device memory: a serving runtime that
has reserved all GPU memory for its own pool, a host program driving the kernels
through a foreign-function interface without a CUDA allocator, or a decode thread
that must not pay cudaMalloc's implicit device synchronisation.  For them the
library keeps the attention partials and row tickets in a fixed array of its own.  These tests
call that entry point through the C ABI twice in a row, on different shapes, and check
each result against the allocating entry point (dsv2_mla_decode with caller buffers) and
against the float64 oracle, to the same 1e-2 relative bound the other attention tests
use: small ragged batches, a 256-row ragged batch whose tile stream fills all 128 CTAs
with many rows cut between CTAs, and 256 rows of one shared position (pos_numel == 1).
They also check that a request larger than the fixed array is refused, and that the
array is usable again after a device error has been read and cleared (clearing zeroes
the row tickets that a launch which gave up could leave behind).

The file name sorts last so that a run stopping at the first failure has already
run every other test.
"""
import ctypes

import pytest
import torch

from oracle import ops as O

pytestmark = pytest.mark.gpu
DEV = "cuda"


def relerr(a, b):
    a, b = a.double().cpu(), b.double().cpu()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))


def _case(B, S, lengths, seed):
    g = torch.Generator().manual_seed(seed)
    cache = torch.randn(B, S, 576, generator=g).to(torch.bfloat16).to(DEV)
    q_abs = torch.randn(B, 16, 512, generator=g).to(torch.bfloat16).to(DEV)
    q_pe = torch.randn(B, 16, 64, generator=g).to(torch.bfloat16).to(DEV)
    pos = (torch.tensor(lengths, dtype=torch.int64) - 1).to(DEV)
    return cache, q_abs, q_pe, pos


def test_noalloc_mla_decode_matches_allocating_entry_point():
    from dsv2 import _lib, ops
    lib = _lib.load()
    torch.cuda.set_device(0)
    scale = 192 ** -0.5
    stream = torch.cuda.current_stream().cuda_stream
    # two calls in a row: the second must not see anything left over from the first
    for B, S, lengths, split in ((3, 700, [613, 5, 700], 64), (4, 300, [300, 64, 65, 1], 128)):
        cache, q_abs, q_pe, pos = _case(B, S, lengths, seed=S + B)
        want = torch.zeros(B, 16, 512, dtype=torch.bfloat16, device=DEV)
        ops.mla_decode(q_abs=q_abs, q_pe=q_pe, cache=cache, positions=pos, softmax_scale=scale,
                       split_len=split, o_lat=want, **ops.mla_workspace(B, S, split, DEV))
        got = torch.full((B, 16, 512), float("nan"), dtype=torch.bfloat16, device=DEV)
        rc = lib.dsv2_mla_decode_noalloc(q_abs.data_ptr(), q_pe.data_ptr(), cache.data_ptr(), cache.stride(0),
                                         S, pos.data_ptr(), pos.numel(), ctypes.c_float(scale), split,
                                         got.data_ptr(), B, stream)
        assert rc == 0, lib.dsv2_last_error().decode()
        torch.cuda.synchronize()
        assert not torch.isnan(got.float()).any()
        assert relerr(got, want) <= 1e-2


def test_noalloc_rejects_requests_larger_than_its_scratch():
    from dsv2 import _lib
    lib = _lib.load()
    t = torch.zeros(16, dtype=torch.bfloat16, device=DEV)
    p = torch.zeros(1, dtype=torch.int64, device=DEV)
    # 5000 rows > the 4096 row tickets of the fixed array
    rc = lib.dsv2_mla_decode_noalloc(t.data_ptr(), t.data_ptr(), t.data_ptr(), 64 * 576, 64, p.data_ptr(), 1,
                                     ctypes.c_float(0.07), 64, t.data_ptr(), 5000, None)
    assert rc == _lib.DSV2_ERR_INVALID
    assert "exceeds" in lib.dsv2_last_error().decode()


def _noalloc(lib, q_abs, q_pe, cache, pos, S, split, B, out):
    rc = lib.dsv2_mla_decode_noalloc(q_abs.data_ptr(), q_pe.data_ptr(), cache.data_ptr(), cache.stride(0), S,
                                     pos.data_ptr(), pos.numel(), ctypes.c_float(192 ** -0.5), split,
                                     out.data_ptr(), B, torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.dsv2_last_error().decode()


@pytest.mark.parametrize("shared_position", [False, True])
def test_noalloc_full_grid_matches_oracle(shared_position):
    from dsv2 import _lib, ops
    lib = _lib.load()
    torch.cuda.set_device(0)
    B, S, split = 256, 1024, 64
    g = torch.Generator().manual_seed(21 + shared_position)
    lengths = [700] * B if shared_position else torch.randint(1, S + 1, (B,), generator=g).tolist()
    cache, q_abs, q_pe, pos = _case(B, S, lengths, seed=99 + shared_position)
    if shared_position:
        pos = pos[:1].contiguous()
    want = torch.zeros(B, 16, 512, dtype=torch.bfloat16, device=DEV)
    ops.mla_decode(q_abs=q_abs, q_pe=q_pe, cache=cache, positions=pos, softmax_scale=192 ** -0.5,
                   split_len=split, o_lat=want, **ops.mla_workspace(B, S, split, DEV))
    ref = O.mla_decode(q_abs.cpu(), q_pe.cpu(), cache.cpu(), torch.tensor(lengths), 192 ** -0.5)
    for _ in range(2):   # the second call reuses the tickets the first one left at zero
        got = torch.full((B, 16, 512), float("nan"), dtype=torch.bfloat16, device=DEV)
        _noalloc(lib, q_abs, q_pe, cache, pos, S, split, B, got)
        torch.cuda.synchronize()
        assert not torch.isnan(got.float()).any()
        assert relerr(got, want) <= 1e-2
        assert relerr(got, ref) <= 1e-2


def test_noalloc_usable_after_a_cleared_device_error():
    from dsv2 import _lib, ops
    lib = _lib.load()
    torch.cuda.set_device(0)
    # an index error (token id outside the vocabulary) sets the device error word
    table = torch.zeros(16, 2048, dtype=torch.bfloat16, device=DEV)
    h = torch.zeros(1, 2048, dtype=torch.bfloat16, device=DEV)
    ops.embed_rmsnorm(torch.tensor([99], dtype=torch.int64, device=DEV), table,
                      torch.ones(2048, dtype=torch.bfloat16, device=DEV), 1e-6, h, torch.zeros_like(h))
    assert _lib.device_error(clear=True) == 2
    assert _lib.device_error(clear=False) == 0
    B, S, lengths = 5, 400, [400, 33, 1, 257, 96]
    cache, q_abs, q_pe, pos = _case(B, S, lengths, seed=7)
    ref = O.mla_decode(q_abs.cpu(), q_pe.cpu(), cache.cpu(), torch.tensor(lengths), 192 ** -0.5)
    for _ in range(2):
        got = torch.full((B, 16, 512), float("nan"), dtype=torch.bfloat16, device=DEV)
        _noalloc(lib, q_abs, q_pe, cache, pos, S, 64, B, got)
        torch.cuda.synchronize()
        assert relerr(got, ref) <= 1e-2
    assert _lib.device_error(clear=False) == 0
