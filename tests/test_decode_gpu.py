"""GPU: paged split-KV decode (with the fused split combine) against the oracle
and the reference goldens; tolerances max-abs 2e-2 / mean-abs 2e-3 on the
bf16 output vs fp32, 1e-3 on the LSE."""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from helpers import (assert_attn_close, build_case, golden_meta, load_attn_golden, oracle_step,
                     to_np32)
from ps_attn import _lib, ops, workloads

pytestmark = pytest.mark.gpu

META = golden_meta()
DECODE_GOLDENS = [n for n, m in META["attention"].items()
                  if "cfg" not in m["spec"] and max(m["spec"]["q_lens"]) == 1]


def run_step(batch, with_lse=True, workspace=None, dtype=None):
    """append + decode on the GPU copy ``batch`` (already on the device)."""
    ops.kv_append(batch.key, batch.value, batch.kv_cache[0], batch.kv_cache[1], batch.slot_mapping)
    out = torch.full_like(batch.q, float("nan"))
    lse = torch.full((batch.q.shape[1], batch.q.shape[0]), float("nan"), dtype=torch.float32,
                     device=batch.q.device) if with_lse else None
    ops.paged_decode(batch.q, batch.kv_cache[0], batch.kv_cache[1], batch.block_table,
                     batch.seq_lens, batch.softmax_scale, out, lse=lse,
                     query_start_loc=batch.query_start_loc, workspace=workspace)
    return out, lse


@pytest.mark.parametrize("name", DECODE_GOLDENS)
def test_decode_matches_reference_golden(cuda_device, name):
    batch = build_case(META["attention"][name]["spec"]).to(cuda_device)
    out, lse = run_step(batch)
    torch.cuda.synchronize()
    gout, glse = load_attn_golden(name)
    assert_attn_close(to_np32(out), gout, to_np32(lse), glse)


def test_decode_config1_shapes_in_bf16(cuda_device):
    # config 1 is fp32 on the CPU; the GPU path runs the same problem in bf16
    batch = workloads.make_config(1, device="cpu", dtype=torch.bfloat16)
    _, (rout, rlse) = oracle_step(batch)
    out, lse = run_step(batch.to(cuda_device))
    torch.cuda.synchronize()
    assert_attn_close(to_np32(out), rout, to_np32(lse), rlse)


@pytest.mark.parametrize("group", [1, 2, 3, 4, 5, 8, 12, 16])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_decode_gqa_groups_and_dtypes(cuda_device, group, dtype):
    hkv = 2
    batch = workloads.make_batch([1] * 5, [1, 15, 16, 17, 333], group * hkv, hkv, dtype=dtype,
                                 seed=100 + group)
    _, (rout, rlse) = oracle_step(batch)
    out, lse = run_step(batch.to(cuda_device))
    torch.cuda.synchronize()
    assert_attn_close(to_np32(out), rout, to_np32(lse), rlse)


@pytest.mark.parametrize("block_size", [16, 32, 64, 256])
def test_decode_block_sizes(cuda_device, block_size):
    batch = workloads.make_batch([1] * 4, [5, 250, 513, 1024], 8, 2, block_size=block_size,
                                 seed=7)
    _, (rout, rlse) = oracle_step(batch)
    out, lse = run_step(batch.to(cuda_device))
    torch.cuda.synchronize()
    assert_attn_close(to_np32(out), rout, to_np32(lse), rlse)


def test_decode_long_and_ragged_forces_splits(cuda_device):
    # one very long sequence among short ones: its (seq, head) segments span many warps
    lens = [9000, 3, 40, 1, 700, 16 * 64]
    batch = workloads.make_batch([1] * len(lens), lens, 8, 4, seed=9)
    _, (rout, rlse) = oracle_step(batch)
    out, lse = run_step(batch.to(cuda_device))
    torch.cuda.synchronize()
    assert_attn_close(to_np32(out), rout, to_np32(lse), rlse)


def test_decode_empty_and_padded_sequences(cuda_device):
    # seq 1 has no cached tokens (q_len 1 -> zero output, lse -inf);
    # seq 3 is a CUDA-graph padding entry (q_len 0): untouched
    batch = workloads.make_batch([1, 1, 1], [50, 1, 20], 4, 2, seed=4).to(cuda_device)
    ops.kv_append(batch.key, batch.value, batch.kv_cache[0], batch.kv_cache[1], batch.slot_mapping)
    seq_lens = torch.tensor([50, 0, 20, 0], dtype=torch.int32, device=cuda_device)
    qsl = torch.tensor([0, 1, 2, 3, 3], dtype=torch.int32, device=cuda_device)
    bt = torch.cat([batch.block_table, batch.block_table[:1]], 0)
    out = torch.full((4, 4, 128), 7.0, dtype=torch.bfloat16, device=cuda_device)
    lse = torch.full((4, 4), 7.0, dtype=torch.float32, device=cuda_device)
    ws = ops.DecodeWorkspace(8, 4, 2, 128, cuda_device)
    ops.paged_decode(batch.q, batch.kv_cache[0], batch.kv_cache[1], bt, seq_lens,
                     batch.softmax_scale, out, lse=lse, query_start_loc=qsl, workspace=ws)
    torch.cuda.synchronize()
    assert ws.status() == 0
    assert (out[1] == 0).all() and torch.isneginf(lse[:, 1]).all()
    assert (out[3] == 7).all() and (lse[:, 3] == 7).all()
    ref_batch = workloads.PagedBatch(**{**batch.__dict__})
    cpu = ref_batch.to("cpu")
    cpu.seq_lens = torch.tensor([50, 0, 20], dtype=torch.int32)
    # oracle on the already-appended cache: disable the second append
    cpu.slot_mapping = torch.full_like(cpu.slot_mapping, -1)
    _, (rout, rlse) = oracle_step(cpu)
    assert_attn_close(to_np32(out[:3]), rout, to_np32(lse[:, :3]), rlse)


def test_decode_no_query_start_loc_and_strided_views(cuda_device):
    # q/out as head-sliced views of a wider buffer, lse as [T, H] transposed view
    batch = workloads.make_batch([1] * 6, [100, 200, 31, 64, 65, 1000], 16, 8, seed=21)
    _, (rout, rlse) = oracle_step(batch)
    g = batch.to(cuda_device)
    ops.kv_append(g.key, g.value, g.kv_cache[0], g.kv_cache[1], g.slot_mapping)
    wide_q = torch.zeros(6, 24, 128, dtype=torch.bfloat16, device=cuda_device)
    wide_q[:, 4:20] = g.q
    wide_o = torch.zeros(6, 20, 128, dtype=torch.bfloat16, device=cuda_device)
    lse_t = torch.zeros(6, 16, dtype=torch.float32, device=cuda_device)
    ops.paged_decode(wide_q[:, 4:20], g.kv_cache[0], g.kv_cache[1], g.block_table, g.seq_lens,
                     g.softmax_scale, wide_o[:, 2:18], lse=lse_t.t())
    torch.cuda.synchronize()
    assert (wide_o[:, :2] == 0).all() and (wide_o[:, 18:] == 0).all()
    assert_attn_close(to_np32(wide_o[:, 2:18]), rout, to_np32(lse_t.t()), rlse)


def test_decode_out_of_range_block_is_flagged(cuda_device):
    batch = workloads.make_batch([1, 1], [40, 40], 4, 2, seed=2).to(cuda_device)
    bt = batch.block_table.clone()
    bt[1, 1] = 10 ** 6
    ws = ops.DecodeWorkspace(4, 4, 2, 128, cuda_device)
    out = torch.empty_like(batch.q)
    ops.paged_decode(batch.q, batch.kv_cache[0], batch.kv_cache[1], bt, batch.seq_lens,
                     batch.softmax_scale, out, workspace=ws)
    torch.cuda.synchronize()
    assert ws.status() & _lib.PS_DEV_BLOCK_OUT_OF_RANGE
    ws.clear_status()
    ops.paged_decode(batch.q, batch.kv_cache[0], batch.kv_cache[1], batch.block_table,
                     batch.seq_lens, batch.softmax_scale, out, workspace=ws)
    torch.cuda.synchronize()
    assert ws.status() == 0


@pytest.mark.parametrize("cfg,max_seqs", [(2, 64), (3, 16), (4, None), (5, 24)])
def test_decode_benchmark_configs(cuda_device, cfg, max_seqs):
    if cfg == 4:  # decode part of the mixed batch
        q_lens, seq_lens, _ = workloads.config_lengths(4)
        batch = workloads.make_batch(q_lens[:128], seq_lens[:128], 32, 8, seed=0)
    else:
        batch = workloads.make_config(cfg, device="cpu", max_seqs=max_seqs)
    _, (rout, rlse) = oracle_step(batch)
    out, lse = run_step(batch.to(cuda_device))
    torch.cuda.synchronize()
    assert_attn_close(to_np32(out), rout, to_np32(lse), rlse)


def test_decode_is_deterministic_and_graph_replayable(cuda_device):
    batch = workloads.make_config(2, device=cuda_device)
    ops.kv_append(batch.key, batch.value, batch.kv_cache[0], batch.kv_cache[1], batch.slot_mapping)
    ws = ops.DecodeWorkspace(batch.num_seqs, 16, 8, 128, cuda_device)
    out1 = torch.empty_like(batch.q)
    ops.paged_decode(batch.q, batch.kv_cache[0], batch.kv_cache[1], batch.block_table,
                     batch.seq_lens, batch.softmax_scale, out1, workspace=ws)
    out2 = torch.empty_like(batch.q)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        ops.paged_decode(batch.q, batch.kv_cache[0], batch.kv_cache[1], batch.block_table,
                         batch.seq_lens, batch.softmax_scale, out2, workspace=ws)
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    out3 = torch.empty_like(batch.q)
    with torch.cuda.graph(graph):
        ops.paged_decode(batch.q, batch.kv_cache[0], batch.kv_cache[1], batch.block_table,
                         batch.seq_lens, batch.softmax_scale, out3, workspace=ws)
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out1, out2) and torch.equal(out1, out3)
    assert ws.status() == 0


def test_decode_full_config2_properties(cuda_device):
    """Full-size config 2: block-table relabelling invariance and a row subset
    against the oracle."""
    batch = workloads.make_config(2, device=cuda_device)
    out, lse = run_step(batch)
    # relabel pages: permute the pool and the table consistently
    nb = batch.kv_cache.shape[1]
    perm = torch.randperm(nb, device=cuda_device, generator=torch.Generator(cuda_device).manual_seed(3))
    inv = torch.empty_like(perm)
    inv[perm] = torch.arange(nb, device=cuda_device)
    kv2 = batch.kv_cache[:, perm].contiguous()   # new block j holds old block perm[j]
    bt2 = inv[batch.block_table.long()].to(torch.int32)
    out2 = torch.empty_like(out)
    lse2 = torch.empty_like(lse)
    ops.paged_decode(batch.q, kv2[0], kv2[1], bt2, batch.seq_lens, batch.softmax_scale, out2,
                     lse=lse2)
    torch.cuda.synchronize()
    assert torch.equal(out, out2) and torch.equal(lse, lse2)
    # oracle on a few rows (CPU cost bounded)
    rows = [0, 17, 63]
    sub = workloads.PagedBatch(**{**batch.__dict__}).to("cpu")
    from oracle import ps_oracle
    kc = sub.kv_cache[0].float().numpy()
    vc = sub.kv_cache[1].float().numpy()
    for r in rows:
        L = int(sub.seq_lens[r])
        kb = ps_oracle.gather_pages(kc, sub.block_table[r].numpy(), L)
        vb = ps_oracle.gather_pages(vc, sub.block_table[r].numpy(), L)
        ro, rl = ps_oracle.attention_ref(to_np32(sub.q[r:r + 1]), kb, vb,
                                         softmax_scale=1 / math.sqrt(128))
        assert_attn_close(to_np32(out[r:r + 1]), ro, to_np32(lse[:, r:r + 1]), rl)


def test_one_workspace_serves_changing_batch_sizes(cuda_device):
    """Regions of calls with different num_seqs must not overlap in a shared
    workspace (counters stay zero between calls)."""
    ws = ops.DecodeWorkspace(64, 16, 8, 128, cuda_device)
    for lens in ([100, 200, 31, 64, 65, 1000], [2049] * 40 + [17] * 24, [5, 4000], [3000] * 64):
        batch = workloads.make_batch([1] * len(lens), lens, 16, 8, seed=len(lens))
        _, (rout, rlse) = oracle_step(batch)
        out, lse = run_step(batch.to(cuda_device), workspace=ws)
        torch.cuda.synchronize()
        assert ws.status() == 0
        assert_attn_close(to_np32(out), rout, to_np32(lse), rlse)


@pytest.mark.parametrize("cfg_lens,heads", [
    ([1, 15, 16, 17, 333, 2049], (16, 8)),
    ([9000, 3, 40, 700], (8, 4)),
    ([100, 200], (32, 2)),
])
def test_fused_append_equals_append_then_decode(cuda_device, cfg_lens, heads):
    """The append fused into the decode launch gives bit-identical outputs and
    cache contents to ps_kv_append followed by the plain decode."""
    hq, hkv = heads
    base = workloads.make_batch([1] * len(cfg_lens), cfg_lens, hq, hkv, seed=55).to(cuda_device)
    a = workloads.PagedBatch(**{**base.__dict__, "kv_cache": base.kv_cache.clone()})
    b = workloads.PagedBatch(**{**base.__dict__, "kv_cache": base.kv_cache.clone()})
    out_a, lse_a = run_step(a)
    out_b = torch.empty_like(b.q)
    lse_b = torch.empty_like(lse_a)
    ws = ops.DecodeWorkspace(len(cfg_lens), hq, hkv, 128, cuda_device)
    ops.paged_decode(b.q, b.kv_cache[0], b.kv_cache[1], b.block_table, b.seq_lens, b.softmax_scale,
                     out_b, lse=lse_b, query_start_loc=b.query_start_loc, workspace=ws,
                     new_key=b.key, new_value=b.value, slot_mapping=b.slot_mapping)
    torch.cuda.synchronize()
    assert ws.status() == 0
    assert torch.equal(out_a, out_b) and torch.equal(lse_a, lse_b)
    assert torch.equal(a.kv_cache, b.kv_cache)


def test_fused_append_padding_and_slot_mismatch(cuda_device):
    batch = workloads.make_batch([1, 1, 1], [40, 17, 64], 8, 2, seed=56).to(cuda_device)
    # padding token (slot -1): nothing appended for sequence 1, attention unchanged
    slots = batch.slot_mapping.clone()
    slots[1] = -1
    ref = workloads.PagedBatch(**{**batch.__dict__, "kv_cache": batch.kv_cache.clone()})
    ops.kv_append(ref.key, ref.value, ref.kv_cache[0], ref.kv_cache[1], slots)
    ref_out = torch.empty_like(ref.q)
    ops.paged_decode(ref.q, ref.kv_cache[0], ref.kv_cache[1], ref.block_table, ref.seq_lens,
                     ref.softmax_scale, ref_out)
    out = torch.empty_like(batch.q)
    ws = ops.DecodeWorkspace(4, 8, 2, 128, cuda_device)
    ops.paged_decode(batch.q, batch.kv_cache[0], batch.kv_cache[1], batch.block_table,
                     batch.seq_lens, batch.softmax_scale, out, workspace=ws, new_key=batch.key,
                     new_value=batch.value, slot_mapping=slots)
    torch.cuda.synchronize()
    assert ws.status() == 0
    assert torch.equal(out, ref_out) and torch.equal(batch.kv_cache, ref.kv_cache)
    # a slot that is not the last position is reported, not silently used
    slots2 = batch.slot_mapping.clone()
    slots2[2] = slots2[0]
    ops.paged_decode(batch.q, batch.kv_cache[0], batch.kv_cache[1], batch.block_table,
                     batch.seq_lens, batch.softmax_scale, out, workspace=ws, new_key=batch.key,
                     new_value=batch.value, slot_mapping=slots2)
    torch.cuda.synchronize()
    assert ws.status() & _lib.PS_DEV_BAD_METADATA

