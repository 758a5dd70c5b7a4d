"""GPU, 2 ranks over NCCL (skipped with fewer than 2 GPUs): KV-head-sharded
append + decode on each GPU with the head outputs all-gathered matches the
single-GPU decode of the unsharded cache (within the decode tolerances: the
split points of the work partition differ, so the fp32 combine order does)."""
from __future__ import annotations

import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, q):
    import datetime
    import sys
    from pathlib import Path

    repo = Path(__file__).resolve().parent.parent
    sys.path.insert(0, str(repo / "prime-rl_b200"))
    import torch.distributed as dist

    from ps_attn import ops, sharding, workloads

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        full = workloads.make_config(5, device="cpu", max_seqs=24)
        shard = sharding.HeadShard(world, rank, 64, 8)
        kv = shard.shard_cache(full.kv_cache).to(dev)
        qd = shard.shard_q(full.q).contiguous().to(dev)
        kd = shard.shard_kv_rows(full.key).contiguous().to(dev)
        vd = shard.shard_kv_rows(full.value).contiguous().to(dev)
        bt, sl, slots = full.block_table.to(dev), full.seq_lens.to(dev), full.slot_mapping.to(dev)
        ops.kv_append(kd, vd, kv[0], kv[1], slots)
        T = full.q.shape[0]
        runner = sharding.HeadShardedDecode(shard, T, 128, qd.dtype, dev)

        def attend(out_local):
            ops.paged_decode(qd, kv[0], kv[1], bt, sl, full.softmax_scale, out_local)

        got = runner.run(attend, T)
        torch.cuda.synchronize()
        if rank == 0:
            q.put(got.cpu())
        dist.barrier()
    except Exception as e:
        q.put(e)
        raise
    finally:
        dist.destroy_process_group()


def test_kv_head_sharded_decode_equals_single_gpu():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    from ps_attn import ops, workloads

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
    if isinstance(got, Exception):
        raise got
    assert all(p.exitcode == 0 for p in procs)
    # single GPU reference: the unsharded batch
    dev = torch.device("cuda", 0)
    full = workloads.make_config(5, device="cpu", max_seqs=24).to(dev)
    ops.kv_append(full.key, full.value, full.kv_cache[0], full.kv_cache[1], full.slot_mapping)
    ref = torch.empty_like(full.q)
    ops.paged_decode(full.q, full.kv_cache[0], full.kv_cache[1], full.block_table, full.seq_lens,
                     full.softmax_scale, ref)
    torch.cuda.synchronize()
    from helpers import assert_attn_close, to_np32

    assert_attn_close(to_np32(got), to_np32(ref))


def _peer_rank(rank, world, port, q, fused=False):
    import datetime
    import sys
    from pathlib import Path

    repo = Path(__file__).resolve().parent.parent
    sys.path.insert(0, str(repo / "prime-rl_b200"))
    import torch.distributed as dist

    from ps_attn import ops, sharding, workloads

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    gth = None
    try:
        full = workloads.make_config(5, device="cpu", max_seqs=24)
        shard = sharding.HeadShard(world, rank, 64, 8)
        T = full.q.shape[0]
        cls = sharding.FusedHeadGather if fused else sharding.PeerHeadGather
        gth = cls.from_process_group(shard, T, torch.bfloat16, device=dev)
        kv = shard.shard_cache(full.kv_cache).to(dev)
        qd = shard.shard_q(full.q).contiguous().to(dev)
        kd = shard.shard_kv_rows(full.key).contiguous().to(dev)
        vd = shard.shard_kv_rows(full.value).contiguous().to(dev)
        bt, sl, slots = full.block_table.to(dev), full.seq_lens.to(dev), full.slot_mapping.to(dev)
        # fused: the append rides in the decode launch (the same rows every call)
        fkw = dict(new_key=kd, new_value=vd, slot_mapping=slots) if fused else {}
        if not fused:
            ops.kv_append(kd, vd, kv[0], kv[1], slots)
        outs = []
        for _ in range(3):  # the same slabs, consecutive calls
            out = torch.full((T, 64, 128), float("nan"), dtype=torch.bfloat16, device=dev)
            gth.decode(qd, kv[0], kv[1], bt, sl, full.softmax_scale, out, **fkw)
            if not fused:
                gth.gather(T, out)
            outs.append(out)
        torch.cuda.synchronize()
        assert int(gth.status.item()) == 0
        assert all(torch.equal(outs[0], o) for o in outs[1:])
        q.put((rank, outs[0].cpu()))
        dist.barrier()
    except Exception as e:
        q.put((rank, e))
        raise
    finally:
        if gth is not None:
            dist.barrier()  # no peer still reads this rank's slab
            gth.close()
        dist.destroy_process_group()


@pytest.mark.parametrize("fused", [False, True], ids=["pull_launch", "fused_into_decode"])
def test_kv_head_sharded_decode_with_peer_head_gather(fused):
    """The same sharded decode with the head outputs exchanged over NVLink
    peer memory instead of NCCL -- pulled by a separate launch
    (ps_head_gather), or stored into the peers by the decode launch itself
    (ps_paged_decode_head_gather, with the append fused too): every rank
    holds the whole output, equal to the single-GPU decode, three calls in a
    row over the same slabs."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    from ps_attn import ops, workloads

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_peer_rank, args=(r, world, port, q, fused)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
    for r in range(world):
        if isinstance(got[r], Exception):
            raise got[r]
    assert all(p.exitcode == 0 for p in procs)
    dev = torch.device("cuda", 0)
    full = workloads.make_config(5, device="cpu", max_seqs=24).to(dev)
    ops.kv_append(full.key, full.value, full.kv_cache[0], full.kv_cache[1], full.slot_mapping)
    ref = torch.empty_like(full.q)
    ops.paged_decode(full.q, full.kv_cache[0], full.kv_cache[1], full.block_table, full.seq_lens,
                     full.softmax_scale, ref)
    torch.cuda.synchronize()
    from helpers import assert_attn_close, to_np32

    for r in range(world):
        assert_attn_close(to_np32(got[r]), to_np32(ref))
