"""The allocation-free latent-attention entry point (dsv2_mla_decode_noalloc).

Some callers of this library cannot allocate device memory: a serving runtime that
has reserved all GPU memory for its own pool, a host program driving the kernels
through a foreign-function interface without a CUDA allocator, or a decode thread
that must not pay cudaMalloc's implicit device synchronisation.  For them the
library keeps the attention partials and row tickets in a fixed array of its own.  This test calls
that entry point through the C ABI twice in a row, on different shapes, and checks
each result against the allocating entry point (dsv2_mla_decode with caller
buffers) to the same 1e-2 relative bound the other attention tests use; it also
checks that a request larger than the fixed array is refused.

The file name sorts last so that a run stopping at the first failure has already
run every other test.
"""
import ctypes

import pytest
import torch

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
