"""GPU: shared-prefix (cascade) plan and decode.

The plan kernel must equal the oracle's plan exactly (integer work).  The
cascade decode must match the fp32 oracle within the attention tolerances
(max-abs 2e-2 / mean-abs 2e-3 on the bf16 output, 1e-3 on the LSE), keep the
fused append bit-exact, fall back to a plain decode on an inconsistent plan,
and share a workspace with plain decodes.
"""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from helpers import assert_attn_close, oracle_step, to_np32
from oracle import ps_oracle
from ps_attn import _lib, ops, workloads

pytestmark = pytest.mark.gpu


def share(batch, groups):
    """Members of each (first, size, blocks) group get the first member's
    leading ``blocks`` block-table entries."""
    bt = batch.block_table.clone()
    for first, size, nb in groups:
        bt[first + 1:first + size, :nb] = bt[first, :nb]
    return workloads.PagedBatch(**{**batch.__dict__, "block_table": bt})


def oracle_plan(batch, min_shared_pages=8, enabled=True):
    return ps_oracle.cascade_plan(batch.block_table.cpu().numpy(), batch.seq_lens.cpu().numpy(),
                                  batch.query_start_loc.cpu().numpy(),
                                  block_size=batch.kv_cache.shape[2],
                                  min_shared_pages=min_shared_pages, enabled=enabled)


def gpu_plan(g, min_shared_pages=8, plan=None):
    return ops.cascade_plan(g.block_table, g.seq_lens, g.q.shape[1], g.kv_cache.shape[3],
                            g.kv_cache.shape[2], query_start_loc=g.query_start_loc,
                            min_shared_pages=min_shared_pages, plan=plan)


def assert_plan_equal(plan, ref):
    v = {k: t.cpu().tolist() for k, t in plan.views().items()}
    n = ref["num_groups"]
    assert v["num_groups"][0] == n
    assert v["seq_group"] == ref["seq_group"]
    assert v["shared_pages"] == ref["shared_pages"]
    assert v["group_first"][:n] == ref["group_first"]
    assert v["group_size"][:n] == ref["group_size"]
    assert v["group_pages"][:n] == ref["group_pages"]


def cascade_step(g, plan, workspace=None, fused=False):
    if not fused:
        ops.kv_append(g.key, g.value, g.kv_cache[0], g.kv_cache[1], g.slot_mapping)
    out = torch.full_like(g.q, float("nan"))
    lse = torch.full((g.q.shape[1], g.q.shape[0]), float("nan"), dtype=torch.float32,
                     device=g.q.device)
    kw = dict(new_key=g.key, new_value=g.value, slot_mapping=g.slot_mapping) if fused else {}
    ops.paged_decode(g.q, g.kv_cache[0], g.kv_cache[1], g.block_table, g.seq_lens,
                     g.softmax_scale, out, lse=lse, query_start_loc=g.query_start_loc,
                     workspace=workspace, cascade=plan, **kw)
    return out, lse


def grouped_batch(hq, hkv, seed, block_size=16, dtype=torch.bfloat16):
    """Groups of 2, 3, 8 and 5 members (prefixes of 70, 9, 64 and 33 pages of
    16 tokens) around single sequences."""
    rng = np.random.default_rng(seed)
    sizes = [(1, 0), (2, 70), (3, 9), (1, 0), (8, 64), (5, 33), (1, 0)]
    lens, groups, b = [], [], 0
    per_block = block_size // 16
    for size, pages in sizes:
        for _ in range(size):
            lens.append(int(pages * 16 + rng.integers(1, 900)))
        if size > 1:
            groups.append((b, size, pages // per_block))
        b += size
    batch = workloads.make_batch([1] * len(lens), lens, hq, hkv, block_size=block_size,
                                 dtype=dtype, seed=seed)
    return share(batch, groups)


@pytest.mark.parametrize("block_size", [16, 32])
def test_plan_kernel_matches_oracle(cuda_device, block_size):
    batch = grouped_batch(16, 4, seed=1, block_size=block_size)
    g = batch.to(cuda_device)
    for mins in (1, 8, 40):
        plan = gpu_plan(g, mins)
        torch.cuda.synchronize()
        assert_plan_equal(plan, oracle_plan(batch, mins))


def test_plan_kernel_on_config3_and_edge_rows(cuda_device):
    batch = workloads.make_config(3, max_seqs=256)
    plan = gpu_plan(batch.to(cuda_device))
    torch.cuda.synchronize()
    ref = oracle_plan(batch)
    assert ref["num_groups"] == 32
    assert_plan_equal(plan, ref)
    # q_len 0 rows and empty sequences break groups; GQA group > 8 gives no plan
    lens = [500, 500, 0, 500, 500, 17, 500]
    b2 = share(workloads.make_batch([1] * 7, lens, 8, 2, seed=9), [(0, 2, 20), (3, 2, 20)])
    g2 = b2.to(cuda_device)
    qsl = torch.tensor([0, 1, 2, 3, 3, 4, 5, 6], dtype=torch.int32, device=cuda_device)
    p2 = ops.cascade_plan(g2.block_table, g2.seq_lens, 8, 2, 16, query_start_loc=qsl)
    torch.cuda.synchronize()
    r2 = ps_oracle.cascade_plan(b2.block_table.numpy(), b2.seq_lens.numpy(), qsl.cpu().numpy())
    assert r2["group_first"] == [0]
    assert_plan_equal(p2, r2)
    p3 = ops.cascade_plan(g2.block_table, g2.seq_lens, 32, 2, 16)
    torch.cuda.synchronize()
    assert p3.views()["num_groups"].item() == 0


@pytest.mark.parametrize("group", [1, 2, 4, 8])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_cascade_decode_matches_oracle(cuda_device, group, dtype):
    hkv = 2
    batch = grouped_batch(group * hkv, hkv, seed=10 + group, dtype=dtype)
    assert oracle_plan(batch)["num_groups"] == 4
    _, (rout, rlse) = oracle_step(batch)
    g = batch.to(cuda_device)
    plan = gpu_plan(g)
    out, lse = cascade_step(g, plan)
    ws = ops.get_workspace(batch.num_seqs, group * hkv, hkv, 128, cuda_device, cascade=True)
    torch.cuda.synchronize()
    assert ws.status() == 0
    assert_attn_close(to_np32(out), rout, to_np32(lse), rlse)


@pytest.mark.parametrize("block_size", [32, 64])
def test_cascade_decode_block_sizes(cuda_device, block_size):
    batch = grouped_batch(32, 8, seed=20, block_size=block_size)
    _, (rout, rlse) = oracle_step(batch)
    g = batch.to(cuda_device)
    out, lse = cascade_step(g, gpu_plan(g))
    torch.cuda.synchronize()
    assert_attn_close(to_np32(out), rout, to_np32(lse), rlse)


@pytest.mark.parametrize("heads", [(16, 4), (16, 2)])
def test_cascade_many_passes_per_group(cuda_device, heads):
    """17 members: 5 passes of 4 members (GQA 4) or 9 passes of 2 (GQA 8)."""
    hq, hkv = heads
    lens = [48 * 16 + 1 + 37 * i for i in range(17)] + [3000, 40]
    batch = share(workloads.make_batch([1] * 19, lens, hq, hkv, seed=21), [(0, 17, 48)])
    _, (rout, rlse) = oracle_step(batch)
    g = batch.to(cuda_device)
    out, lse = cascade_step(g, gpu_plan(g))
    torch.cuda.synchronize()
    assert_attn_close(to_np32(out), rout, to_np32(lse), rlse)


def test_cascade_config3_subset_and_plain_agreement(cuda_device):
    batch = workloads.make_config(3, max_seqs=48)
    _, (rout, rlse) = oracle_step(batch)
    g = batch.to(cuda_device)
    plan = gpu_plan(g)
    out, lse = cascade_step(g, plan)
    ref = workloads.PagedBatch(**{**batch.__dict__}).to(cuda_device)  # fresh cache copy
    ops.kv_append(ref.key, ref.value, ref.kv_cache[0], ref.kv_cache[1], ref.slot_mapping)
    out_p = torch.empty_like(out)
    lse_p = torch.empty_like(lse)
    ops.paged_decode(ref.q, ref.kv_cache[0], ref.kv_cache[1], ref.block_table, ref.seq_lens,
                     ref.softmax_scale, out_p, lse=lse_p, query_start_loc=ref.query_start_loc)
    torch.cuda.synchronize()
    assert_attn_close(to_np32(out), rout, to_np32(lse), rlse)
    assert_attn_close(to_np32(out), to_np32(out_p), to_np32(lse), to_np32(lse_p))


def test_cascade_fused_append_is_bit_identical(cuda_device):
    batch = grouped_batch(32, 8, seed=30)
    a = batch.to(cuda_device)
    b = workloads.PagedBatch(**{**a.__dict__, "kv_cache": a.kv_cache.clone()})
    plan = gpu_plan(a)
    out_a, lse_a = cascade_step(a, plan)
    out_b, lse_b = cascade_step(b, plan, fused=True)
    torch.cuda.synchronize()
    assert torch.equal(out_a, out_b) and torch.equal(lse_a, lse_b)
    assert torch.equal(a.kv_cache, b.kv_cache)


def test_inconsistent_plan_runs_as_plain_decode(cuda_device):
    batch = grouped_batch(16, 4, seed=40)
    _, (rout, rlse) = oracle_step(batch)
    g = batch.to(cuda_device)
    plan = gpu_plan(g)
    v = plan.views()
    v["group_pages"][1] = 10_000  # more pages than its members hold
    ws = ops.DecodeWorkspace(batch.num_seqs, 16, 4, 128, cuda_device, cascade=True)
    out, lse = cascade_step(g, plan, workspace=ws)
    torch.cuda.synchronize()
    assert ws.status() & _lib.PS_DEV_BAD_METADATA
    assert_attn_close(to_np32(out), rout, to_np32(lse), rlse)


def test_workspace_alternates_plain_and_cascade_calls(cuda_device):
    batch = grouped_batch(16, 4, seed=50)
    _, (rout, rlse) = oracle_step(batch)
    g = batch.to(cuda_device)
    ops.kv_append(g.key, g.value, g.kv_cache[0], g.kv_cache[1], g.slot_mapping)
    plan = gpu_plan(g)
    ws = ops.DecodeWorkspace(64, 16, 4, 128, cuda_device, cascade=True)
    for i in range(4):
        out = torch.full_like(g.q, float("nan"))
        lse = torch.full((16, g.q.shape[0]), float("nan"), device=cuda_device)
        ops.paged_decode(g.q, g.kv_cache[0], g.kv_cache[1], g.block_table, g.seq_lens,
                         g.softmax_scale, out, lse=lse, query_start_loc=g.query_start_loc,
                         workspace=ws, cascade=plan if i % 2 else None)
        torch.cuda.synchronize()
        assert ws.status() == 0
        assert_attn_close(to_np32(out), rout, to_np32(lse), rlse)


def test_cascade_plan_and_decode_replay_in_a_graph(cuda_device):
    batch = grouped_batch(32, 8, seed=60)
    g = batch.to(cuda_device)
    ops.kv_append(g.key, g.value, g.kv_cache[0], g.kv_cache[1], g.slot_mapping)
    plan = ops.CascadePlan(64, cuda_device)
    ws = ops.DecodeWorkspace(64, 32, 8, 128, cuda_device, cascade=True)
    out1 = torch.empty_like(g.q)
    gpu_plan(g, plan=plan)
    ops.paged_decode(g.q, g.kv_cache[0], g.kv_cache[1], g.block_table, g.seq_lens,
                     g.softmax_scale, out1, query_start_loc=g.query_start_loc, workspace=ws,
                     cascade=plan)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    out2 = torch.empty_like(g.q)
    with torch.cuda.graph(graph):
        gpu_plan(g, plan=plan)
        ops.paged_decode(g.q, g.kv_cache[0], g.kv_cache[1], g.block_table, g.seq_lens,
                         g.softmax_scale, out2, query_start_loc=g.query_start_loc, workspace=ws,
                         cascade=plan)
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out1, out2) and ws.status() == 0


def test_full_config3_cascade_properties(cuda_device):
    """Full config 3: cascade vs plain decode on every row, oracle on a few."""
    batch = workloads.make_config(3, device=cuda_device)
    ops.kv_append(batch.key, batch.value, batch.kv_cache[0], batch.kv_cache[1], batch.slot_mapping)
    plan = gpu_plan(batch)
    out_c = torch.empty_like(batch.q)
    lse_c = torch.empty(32, batch.num_tokens, device=cuda_device)
    ops.paged_decode(batch.q, batch.kv_cache[0], batch.kv_cache[1], batch.block_table,
                     batch.seq_lens, batch.softmax_scale, out_c, lse=lse_c, cascade=plan)
    out_p = torch.empty_like(out_c)
    lse_p = torch.empty_like(lse_c)
    ops.paged_decode(batch.q, batch.kv_cache[0], batch.kv_cache[1], batch.block_table,
                     batch.seq_lens, batch.softmax_scale, out_p, lse=lse_p)
    torch.cuda.synchronize()
    assert plan.views()["num_groups"].item() == 32
    assert_attn_close(to_np32(out_c), to_np32(out_p), to_np32(lse_c), to_np32(lse_p))
    kc = batch.kv_cache[0].float().cpu().numpy()
    vc = batch.kv_cache[1].float().cpu().numpy()
    bt = batch.block_table.cpu().numpy()
    for r in (0, 7, 130, 255):
        L = int(batch.seq_lens[r])
        kb = ps_oracle.gather_pages(kc, bt[r], L)
        vb = ps_oracle.gather_pages(vc, bt[r], L)
        ro, rl = ps_oracle.attention_ref(to_np32(batch.q[r:r + 1]), kb, vb,
                                         softmax_scale=1 / math.sqrt(128))
        assert_attn_close(to_np32(out_c[r:r + 1]), ro, to_np32(lse_c[:, r:r + 1]), rl)


def test_vllm_impl_forward_with_cascade_plan(cuda_device):
    """PSAttentionImpl.forward (append fused into the decode) with a
    shared-prefix plan in the metadata, as the builder makes it when
    PS_ATTN_CASCADE=1."""
    pytest.importorskip("vllm.v1.attention.backend")
    from ps_attn import backend as psb

    batch = grouped_batch(16, 8, seed=70)
    _, (rout, _) = oracle_step(batch)
    g = batch.to(cuda_device)
    B = batch.num_seqs
    impl = psb.PSAttentionImpl(16, 128, g.softmax_scale, 8, None, None, "auto")
    ws = ops.DecodeWorkspace(B, 16, 8, 128, cuda_device, cascade=True)
    plan = gpu_plan(g)
    md = psb.PSAttentionMetadata(
        num_actual_tokens=B, max_query_len=1, query_start_loc=g.query_start_loc,
        max_seq_len=int(batch.seq_lens.max()), seq_lens=g.seq_lens, block_table=g.block_table,
        slot_mapping=g.slot_mapping, num_decodes=B, num_decode_tokens=B, num_prefills=0,
        workspace=ws, cascade_plan=plan)
    out = torch.empty_like(g.q)
    impl.forward(None, g.q, g.key, g.value, g.kv_cache, md, out)
    torch.cuda.synchronize()
    assert ws.status() == 0 and plan.views()["num_groups"].item() == 4
    assert_attn_close(to_np32(out), rout)
