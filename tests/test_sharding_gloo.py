"""CPU, world_size 2 over gloo: KV-head sharding + head all-gather reproduces
the unsharded oracle; batch balancing keeps GRPO groups whole."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from ps_attn import sharding, workloads


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q_lens, seq_lens, hq, hkv, result_q):
    import sys
    from pathlib import Path

    repo = Path(__file__).resolve().parent.parent
    for p in (repo / "prime-rl_b200", repo, repo / "tests"):
        sys.path.insert(0, str(p))
    from helpers import oracle_step, to_np32  # noqa: F401
    from oracle import ps_oracle

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        full = workloads.make_batch(q_lens, seq_lens, hq, hkv, seed=31)
        shard = sharding.HeadShard(world, rank, hq, hkv)
        kv_local = shard.shard_cache(full.kv_cache)
        q_local = shard.shard_q(full.q)
        key_local = shard.shard_kv_rows(full.key)
        val_local = shard.shard_kv_rows(full.value)
        # local append (oracle byte copy) on the shard
        kc, vc = kv_local[0].clone(), kv_local[1].clone()
        ps_oracle.kv_append(key_local.view(torch.int16).numpy(), val_local.view(torch.int16).numpy(),
                            kc.view(torch.int16).numpy(), vc.view(torch.int16).numpy(),
                            full.slot_mapping.numpy())
        T = full.q.shape[0]
        runner = sharding.HeadShardedDecode(shard, T, 128, torch.float32, "cpu")

        def attend(out_local):
            o, _ = ps_oracle.paged_attention(q_local.float().numpy(), kc.float().numpy(),
                                             vc.float().numpy(), full.block_table.numpy(),
                                             full.seq_lens.numpy(), full.query_start_loc.numpy(),
                                             full.softmax_scale)
            out_local.copy_(torch.from_numpy(o))

        got = runner.run(attend, T)
        if rank == 0:
            result_q.put(got.numpy())
    except Exception as e:  # surface the failure to the parent at once
        result_q.put(e)
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("hq,hkv", [(16, 8), (64, 8), (8, 2)])
def test_head_sharded_decode_matches_unsharded(hq, hkv):
    world = 2
    q_lens = [1, 1, 1]
    seq_lens = [40, 300, 17]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q_lens, seq_lens, hq, hkv, q))
             for r in range(world)]
    for p in procs:
        p.start()
    got = q.get(timeout=240)
    if isinstance(got, Exception):
        raise got
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    import sys
    from pathlib import Path

    sys.path.insert(0, str(Path(__file__).resolve().parent))
    from helpers import oracle_step

    full = workloads.make_batch(q_lens, seq_lens, hq, hkv, seed=31)
    _, (rout, _) = oracle_step(full)
    np.testing.assert_allclose(got, rout, atol=1e-5)


def test_head_shard_ranges_and_errors():
    s = sharding.HeadShard(4, 2, 64, 8)
    assert s.kv_heads == (4, 6) and s.q_heads == (32, 48)
    with pytest.raises(ValueError):
        sharding.HeadShard(3, 0, 64, 8)
    full = torch.arange(2 * 3 * 16 * 8 * 4, dtype=torch.float32).view(2, 3, 16, 8, 4)
    local = s.shard_cache(full)
    assert local.shape == (2, 3, 16, 2, 4) and torch.equal(local, full[:, :, :, 4:6])


def test_balance_sequences_keeps_groups():
    lens = [100, 5000, 300, 20, 7000, 7000, 1, 2]
    parts = sharding.balance_sequences(lens, 2, group_size=2)
    assert sorted(sum(parts, [])) == list(range(8))
    for part in parts:
        for i in part:
            assert (i ^ 1) in part  # both members of a pair together
    loads = [sum(lens[i] for i in p) for p in parts]
    assert max(loads) - min(loads) <= 14000  # LPT: imbalance at most the heaviest group
    parts = sharding.balance_sequences([10, 9, 8, 7, 6, 5], 3)
    assert [sum([10, 9, 8, 7, 6, 5][i] for i in p) for p in parts] == [15, 15, 15]
