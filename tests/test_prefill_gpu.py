"""GPU: tcgen05 chunked prefill (causal, bottom-right, varlen, GQA-packed)
against the reference goldens and the oracle; bf16 output within max-abs
2e-2 / mean-abs 2e-3 of fp32, LSE within 1e-3."""
from __future__ import annotations

import pytest
import torch

from helpers import assert_attn_close, build_case, golden_meta, load_attn_golden, oracle_step, to_np32
from ps_attn import ops, workloads

pytestmark = pytest.mark.gpu

META = golden_meta()


def run_prefill(batch, status=None):
    ops.kv_append(batch.key, batch.value, batch.kv_cache[0], batch.kv_cache[1], batch.slot_mapping)
    out = torch.full_like(batch.q, float("nan"))
    lse = torch.full((batch.q.shape[1], batch.q.shape[0]), float("nan"), dtype=torch.float32,
                     device=batch.q.device)
    ops.chunked_prefill(batch.q, batch.kv_cache[0], batch.kv_cache[1], batch.block_table,
                        batch.seq_lens, batch.query_start_loc, batch.softmax_scale, out, lse=lse,
                        status=status)
    return out, lse


def check_against_oracle(batch, cuda_device):
    _, (rout, rlse) = oracle_step(batch)
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    out, lse = run_prefill(batch.to(cuda_device), status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert_attn_close(to_np32(out), rout, to_np32(lse), rlse)


def test_prefill_matches_reference_golden(cuda_device):
    batch = build_case(META["attention"]["prefill"]["spec"]).to(cuda_device)
    out, lse = run_prefill(batch)
    torch.cuda.synchronize()
    gout, glse = load_attn_golden("prefill")
    assert_attn_close(to_np32(out), gout, to_np32(lse), glse)


@pytest.mark.parametrize("group", [1, 2, 3, 4, 5, 8, 16])
def test_prefill_gqa_groups(cuda_device, group):
    hkv = 2
    q_lens = [1, 7, 64, 130, 33]
    seq_lens = [1, 7 + 100, 64, 130 + 300, 33 + 16]
    batch = workloads.make_batch(q_lens, seq_lens, group * hkv, hkv, seed=200 + group)
    check_against_oracle(batch, cuda_device)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("block_size", [16, 32, 128])
def test_prefill_dtypes_block_sizes(cuda_device, dtype, block_size):
    q_lens = [200, 17, 1]
    seq_lens = [200 + 129, 17 + 511, 1000]
    batch = workloads.make_batch(q_lens, seq_lens, 8, 2, block_size=block_size, dtype=dtype, seed=3)
    check_against_oracle(batch, cuda_device)


def test_prefill_long_chunk_on_context(cuda_device):
    # a config-4 shaped chunk: 2048 causal rows on 1500 cached tokens, Qwen3-4B heads
    batch = workloads.make_batch([2048], [1500 + 2048], 32, 8, seed=44)
    check_against_oracle(batch, cuda_device)


def test_prefill_many_sequences_and_empty_ones(cuda_device):
    q_lens = [3, 0, 1, 50, 0, 129, 128, 127]
    seq_lens = [3, 40, 20, 50 + 77, 0, 129, 128 + 1, 127 + 900]
    batch = workloads.make_batch(q_lens, seq_lens, 16, 4, seed=5)
    check_against_oracle(batch, cuda_device)


def test_prefill_strided_q_and_out_views(cuda_device):
    batch = workloads.make_batch([40, 9], [40 + 60, 9], 8, 2, seed=8)
    _, (rout, rlse) = oracle_step(batch)
    g = batch.to(cuda_device)
    ops.kv_append(g.key, g.value, g.kv_cache[0], g.kv_cache[1], g.slot_mapping)
    T = g.q.shape[0]
    qkv = torch.zeros(T, 8 + 4, 128, dtype=g.q.dtype, device=cuda_device)
    qkv[:, :8] = g.q
    wide_o = torch.zeros(T, 10, 128, dtype=g.q.dtype, device=cuda_device)
    ops.chunked_prefill(qkv[:, :8], g.kv_cache[0], g.kv_cache[1], g.block_table, g.seq_lens,
                        g.query_start_loc, g.softmax_scale, wide_o[:, 1:9])
    torch.cuda.synchronize()
    assert (wide_o[:, 0] == 0).all() and (wide_o[:, 9] == 0).all()
    assert_attn_close(to_np32(wide_o[:, 1:9]), rout)


def test_mixed_batch_through_paged_attention(cuda_device):
    """Decode rows and prefill chunks in one call (the prefill kernel handles
    q_len 1 rows too), checked against the oracle."""
    q_lens, seq_lens, _ = workloads.config_lengths(4)
    # keep it bounded: 16 decodes + 1 prefill chunk of the config-4 shapes
    q_lens = q_lens[:16] + q_lens[128:129]
    seq_lens = seq_lens[:16] + seq_lens[128:129]
    batch = workloads.make_batch(q_lens, seq_lens, 32, 8, seed=0)
    _, (rout, rlse) = oracle_step(batch)
    g = batch.to(cuda_device)
    ops.kv_append(g.key, g.value, g.kv_cache[0], g.kv_cache[1], g.slot_mapping)
    out = torch.empty_like(g.q)
    lse = torch.empty(g.q.shape[1], g.q.shape[0], dtype=torch.float32, device=cuda_device)
    ops.paged_attention(g.q, g.kv_cache[0], g.kv_cache[1], out, g.query_start_loc,
                        g.max_query_len, g.seq_lens, g.softmax_scale, g.block_table, lse=lse)
    torch.cuda.synchronize()
    assert_attn_close(to_np32(out), rout, to_np32(lse), rlse)


def test_vllm_impl_forward_mixed_batch(cuda_device):
    """PSAttentionImpl.forward (which performs the KV append) on a decode-first
    mixed batch."""
    pytest.importorskip("vllm.v1.attention.backend")
    from ps_attn import backend as psb

    q_lens = [1, 1, 1, 37, 200]
    seq_lens = [300, 17, 1024, 37 + 50, 200 + 333]
    batch = workloads.make_batch(q_lens, seq_lens, 16, 8, seed=77)
    _, (rout, _) = oracle_step(batch)
    g = batch.to(cuda_device)
    impl = psb.PSAttentionImpl(16, 128, g.softmax_scale, 8, None, None, "auto")
    ws = ops.DecodeWorkspace(16, 16, 8, 128, cuda_device)
    md = psb.PSAttentionMetadata(
        num_actual_tokens=g.q.shape[0], max_query_len=200, query_start_loc=g.query_start_loc,
        max_seq_len=max(seq_lens), seq_lens=g.seq_lens, block_table=g.block_table,
        slot_mapping=g.slot_mapping, num_decodes=3, num_decode_tokens=3, num_prefills=2,
        workspace=ws)
    out = torch.empty_like(g.q)  # forward appends (decode tokens fused, prefill tokens first)
    impl.forward(None, g.q, g.key, g.value, g.kv_cache, md, out)
    torch.cuda.synchronize()
    assert ws.status() == 0
    assert_attn_close(to_np32(out), rout)


def test_dynamic_unit_claiming_is_bit_identical(cuda_device):
    """ps_chunked_prefill_ws hands the units out through the workspace
    counters; every unit is computed the same way whichever CTA takes it, so
    the result equals the round-robin call's bit for bit, call after call
    (the counters return to zero after each launch)."""
    q_lens, seq_lens, _ = workloads.config_lengths(4)
    q_lens, seq_lens = q_lens[128:132], seq_lens[128:132]  # 4 chunks of 2048 on contexts
    batch = workloads.make_batch(q_lens, seq_lens, 32, 8, seed=12).to(cuda_device)
    ops.kv_append(batch.key, batch.value, batch.kv_cache[0], batch.kv_cache[1], batch.slot_mapping)
    args = (batch.q, batch.kv_cache[0], batch.kv_cache[1], batch.block_table, batch.seq_lens,
            batch.query_start_loc, batch.softmax_scale)
    ref = torch.empty_like(batch.q)
    ref_lse = torch.empty(32, batch.q.shape[0], device=cuda_device)
    ops.chunked_prefill(*args, ref, lse=ref_lse)
    ws = ops.DecodeWorkspace(8, 32, 8, 128, cuda_device)
    for _ in range(3):
        out = torch.full_like(batch.q, float("nan"))
        lse = torch.full_like(ref_lse, float("nan"))
        ops.chunked_prefill(*args, out, lse=lse, workspace=ws)
        torch.cuda.synchronize()
        assert torch.equal(out, ref) and torch.equal(lse, ref_lse)
        assert ws.buffer[16:24].view(torch.int32).tolist() == [0, 0]
