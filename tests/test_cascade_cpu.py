"""CPU: the shared-prefix (cascade) plan rule and the cascade evaluation.

The plan rule is checked on hand-built block tables; the cascade evaluation
(prefix and own pages attended separately, merged with the split combine) must
equal plain attention in fp32 -- the property the GPU cascade decode relies on.
"""
from __future__ import annotations

import numpy as np
import torch

from oracle import ps_oracle
from ps_attn import workloads


def share(batch, groups):
    """Give members of each (first, size, blocks) group the first member's
    leading ``blocks`` block-table entries (what prefix caching produces)."""
    bt = batch.block_table.clone()
    for first, size, nb in groups:
        bt[first + 1:first + size, :nb] = bt[first, :nb]
    return workloads.PagedBatch(**{**batch.__dict__, "block_table": bt})


def plan_of(batch, **kw):
    return ps_oracle.cascade_plan(batch.block_table.numpy(), batch.seq_lens.numpy(),
                                  batch.query_start_loc.numpy(),
                                  block_size=batch.kv_cache.shape[2], **kw)


def test_plan_finds_grpo_groups_of_config3():
    batch = workloads.make_config(3, max_seqs=32)
    plan = plan_of(batch)
    assert plan["num_groups"] == 4
    assert plan["group_first"] == [0, 8, 16, 24]
    assert plan["group_size"] == [8] * 4
    assert plan["group_pages"] == [64] * 4  # the 1024-token prompt
    assert plan["seq_group"] == [b // 8 for b in range(32)]


def test_plan_prefers_tighter_groups_over_a_batch_wide_prompt():
    # 12 sequences share a 20-page system prompt; 3 groups of 4 share 50 pages
    lens = [50 * 16 + 40 + 7 * b for b in range(12)]
    batch = workloads.make_batch([1] * 12, lens, 8, 4, seed=3)
    batch = share(batch, [(0, 12, 20)] + [(4 * i, 4, 50) for i in range(3)])
    plan = plan_of(batch)
    assert plan["group_first"] == [0, 4, 8] and plan["group_size"] == [4, 4, 4]
    assert plan["group_pages"] == [50, 50, 50]
    assert plan["shared_pages"][4] == 20 and plan["shared_pages"][5] == 50


def test_plan_threshold_lengths_and_non_decode_rows():
    lens = [300, 300, 300, 129, 300, 300, 300]
    batch = workloads.make_batch([1] * 7, lens, 8, 2, seed=4)
    batch = share(batch, [(0, 7, 18)])
    plan = plan_of(batch, min_shared_pages=8)
    # page of the last token is never shared: (129 - 1) // 16 = 8 full pages
    assert plan["shared_pages"][3] == 8 and plan["shared_pages"][4] == 8
    # 4 shares more with 5 than with 3: a tighter group starts at 4
    assert plan["group_first"] == [0, 4] and plan["group_pages"] == [8, 18]
    p9 = plan_of(batch, min_shared_pages=9)  # 3 and 4 fall below the threshold
    assert p9["group_first"] == [0, 4] and p9["group_size"] == [3, 3]
    assert p9["group_pages"] == [18, 18] and p9["seq_group"][3] == -1
    # a sequence without exactly one query row never joins a group
    qsl = np.array([0, 1, 2, 2, 3, 4, 5, 6])  # sequence 2 has q_len 0
    p = ps_oracle.cascade_plan(batch.block_table.numpy(), batch.seq_lens.numpy(), qsl)
    assert p["seq_group"][2] == -1 and p["group_first"][0] == 0 and p["group_size"][0] == 2
    assert ps_oracle.cascade_plan(batch.block_table.numpy(), batch.seq_lens.numpy(),
                                  enabled=False)["num_groups"] == 0


def test_plan_counts_pages_within_larger_blocks():
    lens = [32 * 9 + 5, 32 * 9 + 20, 32 * 12]
    batch = workloads.make_batch([1] * 3, lens, 8, 2, block_size=32, seed=5)
    batch = share(batch, [(0, 3, 6)])
    plan = plan_of(batch)
    assert plan["shared_pages"][1:] == [12, 12]  # 6 blocks = 12 pages of 16 tokens
    assert plan["group_pages"] == [12]


def test_cascade_evaluation_equals_plain_attention():
    lens = [1100, 1300, 1025, 2000, 700, 900, 1500]
    batch = workloads.make_batch([1] * 7, lens, 16, 4, seed=6, dtype=torch.float32)
    batch = share(batch, [(0, 4, 64), (4, 3, 40)])
    plan = plan_of(batch)
    assert plan["num_groups"] == 2
    kc = batch.kv_cache[0].numpy()
    vc = batch.kv_cache[1].numpy()
    ro, rl = ps_oracle.paged_attention(batch.q.numpy(), kc, vc, batch.block_table.numpy(),
                                       batch.seq_lens.numpy(), batch.query_start_loc.numpy(),
                                       batch.softmax_scale)
    co, cl = ps_oracle.cascade_decode(batch.q.numpy(), kc, vc, batch.block_table.numpy(),
                                      batch.seq_lens.numpy(), plan, batch.softmax_scale)
    np.testing.assert_allclose(co, ro, atol=2e-6, rtol=0)
    np.testing.assert_allclose(cl, rl, atol=2e-6, rtol=0)
