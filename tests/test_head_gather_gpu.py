"""GPU: the KV-head-sharded decode with its head all-gather over peer memory
(``ps_head_gather``), every rank of a group emulated on one GPU: each rank's
gathered output equals the single-GPU decode of the unsharded batch (within
the decode tolerances: the work partition's split points differ), on the
same slabs for several calls; a peer that never signals makes the bounded
wait report PS_DEV_WAIT_TIMEOUT."""
from __future__ import annotations

import time

import pytest
import torch

from helpers import assert_attn_close, to_np32
from ps_attn import _lib, ops, sharding, workloads

pytestmark = pytest.mark.gpu


def _single_gpu_reference(full, dev):
    g = full.to(dev)
    ops.kv_append(g.key, g.value, g.kv_cache[0], g.kv_cache[1], g.slot_mapping)
    ref = torch.empty_like(g.q)
    ops.paged_decode(g.q, g.kv_cache[0], g.kv_cache[1], g.block_table, g.seq_lens, g.softmax_scale, ref)
    torch.cuda.synchronize()
    return to_np32(ref)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_emulated_peer_head_gather_equals_single_gpu(cuda_device, world):
    hq, hkv = 64, 8
    gathers = sharding.PeerHeadGather.emulated(hq, hkv, world, 24, torch.bfloat16, cuda_device)
    try:
        for step in range(3):  # the same slabs serve consecutive calls
            full = workloads.make_config(5, device="cpu", max_seqs=24, seed=step)
            ref = _single_gpu_reference(full, cuda_device)
            T = full.q.shape[0]
            outs = []
            for r, gth in enumerate(gathers):
                shard = gth.shard
                kv = shard.shard_cache(full.kv_cache).to(cuda_device)
                qd = shard.shard_q(full.q).contiguous().to(cuda_device)
                kd = shard.shard_kv_rows(full.key).contiguous().to(cuda_device)
                vd = shard.shard_kv_rows(full.value).contiguous().to(cuda_device)
                out = torch.full((T, hq, 128), float("nan"), dtype=torch.bfloat16, device=cuda_device)
                gth.decode(qd, kv[0], kv[1], full.block_table.to(cuda_device), full.seq_lens.to(cuda_device),
                           full.softmax_scale, out, new_key=kd, new_value=vd,
                           slot_mapping=full.slot_mapping.to(cuda_device))
                outs.append(out)
            sharding.gather_group(gathers, T, outs)
            torch.cuda.synchronize()
            for gth, out in zip(gathers, outs):
                assert int(gth.status.item()) == 0
                assert_attn_close(to_np32(out), ref)
    finally:
        for g in gathers:
            g.close()


def test_peer_head_gather_wait_runs_out(cuda_device):
    """Rank 0 of a two-rank group gathers alone: barrier 0 gives up after about
    a second, the status word says so, and the context stays usable."""
    gathers = sharding.PeerHeadGather.emulated(16, 8, 2, 4, torch.bfloat16, cuda_device)
    try:
        out = torch.zeros(4, 16, 128, dtype=torch.bfloat16, device=cuda_device)
        t0 = time.monotonic()
        gathers[0].gather(4, out)
        torch.cuda.synchronize()
        dt = time.monotonic() - t0
        assert int(gathers[0].status.item()) & _lib.PS_DEV_WAIT_TIMEOUT
        assert 0.9 < dt < 10.0
        assert float((torch.ones(4, device=cuda_device) * 2).sum()) == 8.0
    finally:
        for g in gathers:
            g.close()
