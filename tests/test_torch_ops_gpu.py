"""GPU: ``torch.ops.ps_attn.*`` run the library's kernels (same bytes as the
Python API) and pass ``torch.library.opcheck`` (schema mutations, fake
implementation, autograd registration)."""
from __future__ import annotations

import pytest
import torch

from ps_attn import ops, torch_ops, workloads

pytestmark = pytest.mark.gpu

CHECKS = ("test_schema", "test_faketensor", "test_autograd_registration")


def test_kv_append_op(cuda_device):
    b = workloads.make_config(2, device=cuda_device, max_seqs=8)
    kc1, vc1 = b.kv_cache[0].clone(), b.kv_cache[1].clone()
    kc2, vc2 = kc1.clone(), vc1.clone()
    ops.kv_append(b.key, b.value, kc1, vc1, b.slot_mapping)
    torch.ops.ps_attn.kv_append(b.key, b.value, kc2, vc2, b.slot_mapping)
    torch.cuda.synchronize()
    assert torch.equal(kc1.view(torch.int16), kc2.view(torch.int16))
    assert torch.equal(vc1.view(torch.int16), vc2.view(torch.int16))
    torch.library.opcheck(torch.ops.ps_attn.kv_append.default, (b.key, b.value, kc2, vc2, b.slot_mapping),
                          test_utils=CHECKS)


def test_paged_decode_op_with_fused_append(cuda_device):
    b = workloads.make_config(2, device=cuda_device, max_seqs=16)
    B, hq = b.num_seqs, b.q.shape[1]
    cache_a, cache_b = b.kv_cache.clone(), b.kv_cache.clone()
    out_a, out_b = torch.empty_like(b.q), torch.empty_like(b.q)
    lse_a = torch.empty(hq, B, dtype=torch.float32, device=cuda_device)
    lse_b = torch.empty_like(lse_a)
    ops.paged_decode(b.q, cache_a[0], cache_a[1], b.block_table, b.seq_lens, b.softmax_scale, out_a, lse=lse_a,
                     query_start_loc=b.query_start_loc, workspace=ops.DecodeWorkspace(B, hq, 8, 128, cuda_device),
                     new_key=b.key, new_value=b.value, slot_mapping=b.slot_mapping)
    ws = torch_ops.workspace_tensor(B, hq, 8, device=cuda_device)
    args = (b.q, cache_b[0], cache_b[1], b.block_table, b.seq_lens, b.query_start_loc, b.softmax_scale,
            b.max_seq_len, out_b, lse_b, ws, b.key, b.value, b.slot_mapping)
    torch.ops.ps_attn.paged_decode(*args)
    torch.cuda.synchronize()
    assert torch.equal(out_a, out_b) and torch.equal(lse_a, lse_b)
    assert torch.equal(cache_a.view(torch.int16), cache_b.view(torch.int16))
    torch.library.opcheck(torch.ops.ps_attn.paged_decode.default, args, test_utils=CHECKS)


def test_chunked_prefill_op(cuda_device):
    q_lens, ctx = [100, 7, 300], [50, 0, 1000]
    b = workloads.make_batch(q_lens, [c + q for c, q in zip(ctx, q_lens)], 32, 8, seed=5, device=cuda_device)
    ops.kv_append(b.key, b.value, b.kv_cache[0], b.kv_cache[1], b.slot_mapping)
    out_a, out_b = torch.empty_like(b.q), torch.empty_like(b.q)
    lse_a = torch.empty(32, b.num_tokens, dtype=torch.float32, device=cuda_device)
    lse_b = torch.empty_like(lse_a)
    ops.chunked_prefill(b.q, b.kv_cache[0], b.kv_cache[1], b.block_table, b.seq_lens, b.query_start_loc,
                        b.softmax_scale, out_a, lse=lse_a)
    ws = torch_ops.workspace_tensor(b.num_seqs, 32, 8, device=cuda_device)
    args = (b.q, b.kv_cache[0], b.kv_cache[1], b.block_table, b.seq_lens, b.query_start_loc, b.softmax_scale,
            b.max_seq_len, out_b, lse_b, ws)
    torch.ops.ps_attn.chunked_prefill(*args)
    torch.cuda.synchronize()
    # dynamic unit claiming (workspace) and the static round-robin give identical bytes
    assert torch.equal(out_a, out_b) and torch.equal(lse_a, lse_b)
    torch.library.opcheck(torch.ops.ps_attn.chunked_prefill.default, args, test_utils=CHECKS)
