"""Failure detection on one GPU, without faulting it.

Every wait in the library is bounded and every index it reads is checked; a failure sets
the device error word and the kernel skips the work instead of trapping.  These tests make
those paths run on purpose, with nothing that can fault or hang the GPU:
  * the cross-GPU waits of expert parallelism, on a two-rank peer table whose second
    "rank" is a local buffer that nobody signals (poll limit set short through
    dsv2_peer_table.wait_polls): the wait gives up, the error word reads
    DSV2_DEVERR_TIMEOUT, dsv2_stream_check reports DSV2_ERR_DEVICE, and once the missing
    arrival is supplied by the host the same call completes with the right routing;
  * token ids outside the vocabulary and positions outside the cache: DSV2_DEVERR_INDEX,
    nothing written out of bounds;
  * the engine's recovery: after a step with an error, recover() returns the code,
    clears it and zeroes the progress counters (poisoned here by the host, as a launch
    that gave up would leave them), and the next step matches a fresh engine bit for bit.
"""
import time

import pytest
import torch

from oracle import ops as O

pytestmark = pytest.mark.gpu
DEV = "cuda"
TIMEOUT, INDEX = 1, 2


@pytest.fixture(autouse=True)
def clean_error_word():
    from dsv2 import _lib
    torch.cuda.synchronize()
    _lib.device_error(clear=True)
    yield
    torch.cuda.synchronize()
    _lib.device_error(clear=True)


def _peer_table(B, polls):
    """World-2 table over two local buffers (rank 0 = this process; rank 1 never runs)."""
    from dsv2 import _lib
    H = 2048

    def up(n):
        return (n + 255) // 256 * 256
    off_xg = 0
    off_ids = up(2 * B * H * 2)
    off_w = up(off_ids + 2 * B * 6 * 4)
    off_part = up(off_w + 2 * B * 6 * 4)
    off_ctr = up(off_part + B * 8 * H * 4)
    total = off_ctr + 256
    bufs = [torch.zeros(total, dtype=torch.uint8, device=DEV) for _ in range(2)]
    epoch = torch.zeros(1, dtype=torch.int64, device=DEV)
    t = _lib.PeerTable()
    t.world, t.rank = 2, 0
    t.base[0], t.base[1] = bufs[0].data_ptr(), bufs[1].data_ptr()
    t.xg_offset, t.ids_offset, t.w_offset, t.part_offset, t.ctr_offset = off_xg, off_ids, off_w, off_part, off_ctr
    t.rows_per_rank, t.n_moe_layers = B, 1
    t.epoch = epoch.data_ptr()
    t.wait_polls = polls
    views = {
        "xg": bufs[0][off_xg:off_xg + 2 * B * H * 2].view(torch.bfloat16).view(2 * B, H),
        "ids": bufs[0][off_ids:off_ids + 2 * B * 24].view(torch.int32).view(2 * B, 6),
        "w": bufs[0][off_w:off_w + 2 * B * 24].view(torch.float32).view(2 * B, 6),
        "part": bufs[0][off_part:off_part + B * 8 * H * 4].view(torch.float32).view(B, 8, H),
        "ctr": bufs[0][off_ctr:off_ctr + 256].view(torch.int64),   # [0] dispatch, [16] combine
    }
    return t, bufs, epoch, views


def test_peer_waits_give_up_and_complete_once_signalled():
    from dsv2 import _lib, ops
    B, E = 8, 64
    t, bufs, epoch, v = _peer_table(B, polls=4096)
    g = torch.Generator().manual_seed(3)
    x = torch.randn(B, 2048, generator=g).to(torch.bfloat16).to(DEV)
    gate = (0.02 * torch.randn(E, 2048, generator=g)).to(torch.bfloat16).to(DEV)
    logits = torch.zeros(B, E, device=DEV)
    ids32 = torch.zeros(B, 6, dtype=torch.int32, device=DEV)
    w = torch.zeros(B, 6, device=DEV)
    ids64 = torch.zeros(B, 6, dtype=torch.int64, device=DEV)
    # dispatch: this rank's rows go to both buffers, one arrival per buffer
    ops.router(x=x, w=gate, scaling=1.0, logits=logits, topk_ids32=ids32, topk_weights=w, topk_ids64=ids64,
               peers=t, row_base=0)
    torch.cuda.synchronize()
    assert int(v["ctr"][0]) == 1 and _lib.device_error(clear=False) == 0
    go = torch.full((32 + 3,), -1, dtype=torch.int32, device=DEV)
    rt = torch.zeros(16 * 8, dtype=torch.int32, device=DEV)
    rs, rw = torch.zeros_like(rt), torch.zeros(16 * 8, device=DEV)
    xs = torch.zeros(16 * 8, 2048, dtype=torch.bfloat16, device=DEV)

    def bucket():
        ops.moe_bucket(v["ids"], v["w"], 0, 32, 0, B, go, rt, rs, rw, gather_src=v["xg"], gather_out=xs,
                       peers=t, moe_layer=0)
    # bucketing waits for rank 1's dispatch, which never comes: it gives up, bounded
    t0 = time.perf_counter()
    bucket()
    with pytest.raises(_lib.Dsv2Error) as ei:
        _lib.stream_check(ops.stream())
    assert "device error word 1" in str(ei.value)
    assert time.perf_counter() - t0 < 5.0
    assert int((go != -1).sum()) == 0            # the kernel skipped its work
    assert _lib.device_error(clear=True) == TIMEOUT
    assert _lib.device_error(clear=False) == 0
    # the combine wait of the next add+RMSNorm gives up the same way
    h = torch.zeros(B, 2048, dtype=torch.bfloat16, device=DEV)
    y = torch.zeros_like(h)
    ops.add_rmsnorm(h, v["part"], torch.ones(2048, dtype=torch.bfloat16, device=DEV), 1e-6, y,
                    peers=t, moe_layer=0)
    torch.cuda.synchronize()
    assert _lib.device_error(clear=True) == TIMEOUT
    # rank 1's arrival supplied by the host (its rows: a copy of rank 0's): the same call
    # now completes and buckets both ranks' rows like the oracle
    v["xg"][B:] = v["xg"][:B]
    v["ids"][B:] = v["ids"][:B]
    v["w"][B:] = v["w"][:B]
    v["ctr"][0] += 1
    bucket()
    _lib.stream_check(ops.stream())
    e_go, e_rt, e_rs, e_rw = O.bucket(v["ids"].cpu(), v["w"].cpu(), 0, 32, 0, B)
    assert torch.equal(go.cpu(), e_go)
    n = int(e_go[-1])
    assert torch.equal(rt.cpu()[:n], e_rt) and torch.equal(rs.cpu()[:n], e_rs)
    assert torch.equal(xs[:n].cpu(), v["xg"].cpu()[e_rt.long()])
    # the router's own routing equals the oracle's
    _, ids_ref, _ = O.router(x.cpu(), gate.cpu(), 1.0)
    assert all(set(a) == set(b) for a, b in zip(ids64.cpu().tolist(), ids_ref.tolist()))


def test_token_id_outside_the_vocabulary_is_flagged():
    from dsv2 import _lib, ops
    V, C = 1000, 2048
    g = torch.Generator().manual_seed(5)
    table = torch.randn(V, C, generator=g).to(torch.bfloat16).to(DEV)
    w = torch.ones(C, dtype=torch.bfloat16, device=DEV)
    ids = torch.tensor([7, V, -3, V - 1], dtype=torch.int64, device=DEV)
    h = torch.zeros(4, C, dtype=torch.bfloat16, device=DEV)
    y = torch.zeros_like(h)
    ops.embed_rmsnorm(ids, table, w, 1e-6, h, y)
    torch.cuda.synchronize()
    assert _lib.device_error(clear=True) == INDEX
    assert torch.equal(h[0], table[7]) and torch.equal(h[3], table[V - 1])
    assert torch.equal(h[1], table[0]) and torch.equal(h[2], table[0])   # bad ids read row 0


def test_position_outside_the_cache_is_flagged():
    from dsv2 import _lib, ops
    B, S = 3, 40
    g = torch.Generator().manual_seed(6)
    qkva = torch.randn(B, 3648, generator=g).to(torch.bfloat16).to(DEV)
    cache = torch.zeros(B, S, 576, dtype=torch.bfloat16, device=DEV)
    cos = torch.ones(S, 32, device=DEV)
    sin = torch.zeros(S, 32, device=DEV)
    q_pe = torch.zeros(B, 16, 64, dtype=torch.bfloat16, device=DEV)
    pos = torch.tensor([5, S, 1 << 40], dtype=torch.int64, device=DEV)
    ops.mla_prep(qkva=qkva, kv_norm_w=torch.ones(512, dtype=torch.bfloat16, device=DEV), eps=1e-6, cos=cos,
                 sin=sin, positions=pos, cache=cache, q_pe_out=q_pe)
    torch.cuda.synchronize()
    assert _lib.device_error(clear=True) == INDEX
    assert float(cache[0, 5].abs().sum()) > 0                 # the valid row was written
    assert float(cache[1:].abs().sum()) == 0                  # nothing else was


def test_engine_recovers_after_a_device_error():
    from dsv2 import _lib
    from dsv2.engine import DecodeEngine
    from oracle.hf_model import build_model, dsv2_lite_config
    model = build_model(dsv2_lite_config(num_layers=2), seed=1, device=DEV, dtype=torch.bfloat16)
    g = torch.Generator().manual_seed(8)
    prompts = [torch.randint(0, 102400, (n,), generator=g) for n in (12, 30, 7, 21)]
    engines = []
    for _ in range(2):
        eng = DecodeEngine(model, batch=4, max_len=64, family="batch", keep_logits=True)
        eng.prefill(prompts)
        engines.append(eng)
    eng, fresh = engines
    assert eng.recover() == 0
    # a step fed an id outside the vocabulary: flagged, the row reads embedding row 0
    ids = eng.input_ids.clone()
    eng.input_ids[1] = 102400 + 5
    eng.step()
    # progress counters as a launch that gave up would leave them
    eng.moe_sync.fill_(3)
    eng.mla_sync.fill_(1)
    assert eng.recover() == INDEX
    assert int(eng.moe_sync.abs().sum()) == 0 and int(eng.mla_sync.abs().sum()) == 0
    assert _lib.device_error(clear=False) == 0
    # rolled back to the prefill state, the next steps equal a fresh engine's, bit for bit
    eng.restore()
    assert torch.equal(eng.input_ids, ids)
    for _ in range(2):
        eng.step()
        fresh.step()
        torch.cuda.synchronize()
        assert torch.equal(eng.next_ids, fresh.next_ids)
        assert torch.equal(eng.logits, fresh.logits)
    assert eng.recover() == 0
