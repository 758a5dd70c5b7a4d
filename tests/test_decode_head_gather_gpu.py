"""GPU, one device: the decode with the head all-gather fused in
(``ps_paged_decode_head_gather``), checked without a second GPU.

* World 1: the launch equals ``ps_paged_decode`` bit for bit and its closing
  barriers run against itself; two calls in a row.
* World 2 (16-bit and fp8 caches), rank 0 alone, rank 1 played by the test:
  rank 1's "rows written" and "rows copied" flags are set in rank 0's slab
  before the call (a peer that already finished) and its rows pre-filled in
  rank 0's slab.  The pushed rows (from the combine and, for segments one
  warp streams alone, from the transposed accumulators) must equal the plain
  decode's bit for bit.  The
  launch must store rank 0's rows into rank 1's slab (plain device memory
  here), copy rank 1's rows into ``out``, publish its own flags in both slabs
  and advance rank 0's epoch -- two calls in a row.
* World 2 with a peer that never signals: the bounded wait gives up after
  about a second with PS_DEV_WAIT_TIMEOUT in the status word (no hang), and
  rank 0's own rows are still correct.

The real two-GPU exchange is ``tests/test_sharded_decode_multigpu.py``.
"""
from __future__ import annotations

import pytest
import torch

from ps_attn import _lib, ops, sharding, workloads
from ps_attn.peer import PeerSlabs

pytestmark = pytest.mark.gpu

HQ_ALL, HKV_ALL = 64, 8


def _slabs(world, rank, max_tokens, dev):
    nbytes = sharding.FusedHeadGather.slab_bytes(max_tokens, HQ_ALL)
    bufs = [torch.zeros(nbytes, dtype=torch.uint8, device=dev) for _ in range(world)]
    view = PeerSlabs(world, rank, nbytes, [b.data_ptr() for b in bufs], dev)
    return bufs, view


def _words(buf):
    return buf[:256].view(torch.int32)


def _rows(buf, max_tokens):
    return buf[256:256 + max_tokens * HQ_ALL * 256].view(torch.bfloat16).view(max_tokens, HQ_ALL, 128)


def _shard_batch(world, dev, seed=5, fp8=False):
    """Config-5-shaped sequences, this rank's heads only (rank 0 of `world`);
    fp8: the cache as e4m3 codes with per-tensor scales (``b.skw``)."""
    lens = [2048, 17, 1, 4000, 333, 16, 9000, 1025, 64, 31]
    hq, hkv = HQ_ALL // world, HKV_ALL // world
    b = workloads.make_batch([1] * len(lens), lens, hq, hkv, seed=seed, device=dev)
    ops.kv_append(b.key, b.value, b.kv_cache[0], b.kv_cache[1], b.slot_mapping)
    b.skw = {}
    if fp8:
        ks = torch.tensor(0.03, dtype=torch.float32, device=dev)
        vs = torch.tensor(0.02, dtype=torch.float32, device=dev)
        b.kv_cache = torch.stack([(b.kv_cache[0].float() / ks).to(torch.float8_e4m3fn).view(torch.uint8),
                                  (b.kv_cache[1].float() / vs).to(torch.float8_e4m3fn).view(torch.uint8)])
        b.skw = dict(k_scale=ks, v_scale=vs)
    return b


def _plain(b):
    out = torch.empty_like(b.q)
    lse = torch.empty(b.q.shape[1], b.q.shape[0], dtype=torch.float32, device=b.q.device)
    ops.paged_decode(b.q, b.kv_cache[0], b.kv_cache[1], b.block_table, b.seq_lens, b.softmax_scale, out,
                     lse=lse, query_start_loc=b.query_start_loc, **b.skw)
    return out, lse


def _fused(gth, b, out, lse):
    gth.decode(b.q, b.kv_cache[0], b.kv_cache[1], b.block_table, b.seq_lens, b.softmax_scale, out,
               lse=lse, query_start_loc=b.query_start_loc, **b.skw)


def test_world_one_equals_plain_decode(cuda_device):
    b = _shard_batch(1, cuda_device)
    T = b.q.shape[0]
    ref, ref_lse = _plain(b)
    bufs, view = _slabs(1, 0, T, cuda_device)
    gth = sharding.FusedHeadGather(sharding.HeadShard(1, 0, HQ_ALL, HKV_ALL), T, torch.bfloat16, view,
                                   torch.zeros(1, dtype=torch.int32, device=cuda_device))
    for call in (1, 2):
        out = torch.full((T, HQ_ALL, 128), float("nan"), dtype=torch.bfloat16, device=cuda_device)
        lse = torch.full_like(ref_lse, float("nan"))
        _fused(gth, b, out, lse)
        torch.cuda.synchronize()
        assert int(gth.status.item()) == 0
        assert torch.equal(out.view(torch.int16), ref.view(torch.int16))
        assert float((lse - ref_lse).abs().max()) <= 1e-5
        assert int(_words(bufs[0])[32]) == call  # calls completed


@pytest.mark.parametrize("fp8", [False, True], ids=["bf16_cache", "fp8_cache"])
def test_world_two_rank_zero_with_a_finished_peer(cuda_device, fp8):
    world = 2
    b = _shard_batch(world, cuda_device, fp8=fp8)
    T, hq = b.q.shape[0], HQ_ALL // world
    ref, ref_lse = _plain(b)
    bufs, view = _slabs(world, 0, T, cuda_device)
    gth = sharding.FusedHeadGather(sharding.HeadShard(world, 0, HQ_ALL, HKV_ALL), T, torch.bfloat16, view,
                                   torch.zeros(1, dtype=torch.int32, device=cuda_device))
    g = torch.Generator().manual_seed(11)
    for call in (1, 2):
        # rank 1: its rows in rank 0's slab, both of its flags for this call
        peer_rows = torch.randn(T, hq, 128, generator=g).to(torch.bfloat16).to(cuda_device)
        _rows(bufs[0], T)[:, hq:] = peer_rows
        _words(bufs[0])[0 * 8 + 1] = call
        _words(bufs[0])[1 * 8 + 1] = call
        out = torch.full((T, HQ_ALL, 128), float("nan"), dtype=torch.bfloat16, device=cuda_device)
        lse = torch.full_like(ref_lse, float("nan"))
        _fused(gth, b, out, lse)
        torch.cuda.synchronize()
        assert int(gth.status.item()) == 0
        # rank 0's heads computed here, rank 1's copied from the slab
        assert torch.equal(out[:, :hq].view(torch.int16), ref.view(torch.int16))
        assert torch.equal(out[:, hq:].view(torch.int16), peer_rows.view(torch.int16))
        assert float((lse - ref_lse).abs().max()) <= 1e-5
        # rank 0's rows stored into rank 1's slab, flags published in both slabs
        assert torch.equal(_rows(bufs[1], T)[:, :hq].view(torch.int16), ref.view(torch.int16))
        for buf in bufs:
            assert int(_words(buf)[0 * 8 + 0]) == call and int(_words(buf)[1 * 8 + 0]) == call
        assert int(_words(bufs[0])[32]) == call


def test_world_two_peer_never_signals_times_out(cuda_device):
    world = 2
    b = _shard_batch(world, cuda_device, seed=6)
    T, hq = b.q.shape[0], HQ_ALL // world
    ref, _ = _plain(b)
    bufs, view = _slabs(world, 0, T, cuda_device)
    gth = sharding.FusedHeadGather(sharding.HeadShard(world, 0, HQ_ALL, HKV_ALL), T, torch.bfloat16, view,
                                   torch.zeros(1, dtype=torch.int32, device=cuda_device))
    out = torch.zeros(T, HQ_ALL, 128, dtype=torch.bfloat16, device=cuda_device)
    _fused(gth, b, out, None)
    torch.cuda.synchronize()
    assert int(gth.status.item()) & _lib.PS_DEV_WAIT_TIMEOUT
    assert torch.equal(out[:, :hq].view(torch.int16), ref.view(torch.int16))
    assert torch.equal(out[:, hq:], torch.zeros_like(out[:, hq:]))  # nothing copied


def test_rows_past_the_slabs_are_refused(cuda_device):
    """A query row index >= the gather's num_tokens is reported
    (PS_DEV_BAD_METADATA) and not stored into a peer's slab."""
    world = 1
    b = _shard_batch(world, cuda_device, seed=7)
    T = b.q.shape[0]
    bufs, view = _slabs(world, 0, T, cuda_device)
    gth = sharding.FusedHeadGather(sharding.HeadShard(world, 0, HQ_ALL, HKV_ALL), T, torch.bfloat16, view,
                                   torch.zeros(1, dtype=torch.int32, device=cuda_device))
    qsl = b.query_start_loc + T  # rows T..2T-1: in q and out, past the slabs' T rows
    q = torch.cat([b.q, b.q])
    out = torch.zeros(2 * T, HQ_ALL, 128, dtype=torch.bfloat16, device=cuda_device)
    hp = gth._problem(T, out)
    ops.paged_decode(q, b.kv_cache[0], b.kv_cache[1], b.block_table, b.seq_lens, b.softmax_scale,
                     out[:, :HQ_ALL], query_start_loc=qsl, head_gather=hp)
    torch.cuda.synchronize()
    assert int(gth.status.item()) & _lib.PS_DEV_BAD_METADATA
