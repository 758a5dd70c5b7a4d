"""GPU: parity with the reference's own GPU attention -- vLLM's FA4 path as
its FlashAttention backend calls it on sm_100
(``vllm/v1/attention/backends/flash_attn.py:796-817``: ``reshape_and_cache_flash``
then ``flash_attn_varlen_func(..., block_table, seqused_k, fa_version=4)``),
run as a black box on the same seeded inputs.

Both sides round fp32 accumulators to bf16/fp16 once, so the bars are the
bf16 attention tolerances (max-abs 2e-2, mean-abs 2e-3) and LSE 1e-3, and the
caches after the append must be bit-identical.
"""
from __future__ import annotations

import pytest
import torch

from helpers import LSE_ABS, OUT_MAX_ABS, OUT_MEAN_ABS
from ps_attn import ops, workloads

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def fa4():
    try:
        from vllm import _custom_ops as vops
        from vllm.vllm_flash_attn.flash_attn_interface import flash_attn_varlen_func
    except ImportError as e:  # the image ships vLLM; a missing build is a test environment gap
        pytest.skip(f"vLLM FA4 unavailable: {e}")
    return vops, flash_attn_varlen_func


def fa4_step(fa4, batch, key_cache, value_cache):
    """The reference's append + attention over (copies of) the batch's cache."""
    vops, flash_attn_varlen_func = fa4
    ones = torch.ones(1, dtype=torch.float32, device=batch.q.device)
    vops.reshape_and_cache_flash(batch.key, batch.value, key_cache, value_cache, batch.slot_mapping,
                                 "auto", ones, ones)
    out = torch.empty_like(batch.q)
    _, lse = flash_attn_varlen_func(
        q=batch.q, k=key_cache, v=value_cache, out=out, cu_seqlens_q=batch.query_start_loc,
        max_seqlen_q=batch.max_query_len, seqused_k=batch.seq_lens, max_seqlen_k=batch.max_seq_len,
        softmax_scale=batch.softmax_scale, causal=True, block_table=batch.block_table, softcap=0.0,
        fa_version=4, num_splits=0, return_softmax_lse=True)
    return out, lse


def ours_step(batch):
    """ps_attn's path for the same batch: decode rows with the append fused,
    prefill tokens appended then attended by the tcgen05 prefill kernel."""
    kc, vc = batch.kv_cache[0], batch.kv_cache[1]
    qlens = (batch.query_start_loc[1:] - batch.query_start_loc[:-1]).tolist()
    nd = 0
    while nd < len(qlens) and qlens[nd] == 1:
        nd += 1
    T = batch.num_tokens
    out = torch.full_like(batch.q, float("nan"))
    lse = torch.full((batch.q.shape[1], T), float("nan"), dtype=torch.float32, device=batch.q.device)
    ntok = int(batch.query_start_loc[nd])
    if nd < len(qlens):
        ops.kv_append(batch.key[ntok:], batch.value[ntok:], kc, vc, batch.slot_mapping[ntok:])
    if nd > 0:
        ops.paged_decode(batch.q[:ntok], kc, vc, batch.block_table[:nd], batch.seq_lens[:nd],
                         batch.softmax_scale, out[:ntok], lse=lse[:, :ntok],
                         query_start_loc=batch.query_start_loc[:nd + 1], new_key=batch.key,
                         new_value=batch.value, slot_mapping=batch.slot_mapping)
    if nd < len(qlens):
        ops.chunked_prefill(batch.q, kc, vc, batch.block_table[nd:], batch.seq_lens[nd:],
                            batch.query_start_loc[nd:], batch.softmax_scale, out, lse=lse)
    return out, lse


def compare(fa4, batch):
    kc_ref, vc_ref = batch.kv_cache[0].clone(), batch.kv_cache[1].clone()
    out_ref, lse_ref = fa4_step(fa4, batch, kc_ref, vc_ref)
    out, lse = ours_step(batch)
    torch.cuda.synchronize()
    # the append: bit-identical caches
    assert torch.equal(batch.kv_cache[0].view(torch.int16), kc_ref.view(torch.int16))
    assert torch.equal(batch.kv_cache[1].view(torch.int16), vc_ref.view(torch.int16))
    assert torch.isfinite(out).all()
    err = (out.float() - out_ref.float()).abs()
    assert float(err.max()) <= OUT_MAX_ABS, f"max abs {float(err.max()):.3e}"
    assert float(err.mean()) <= OUT_MEAN_ABS, f"mean abs {float(err.mean()):.3e}"
    d = (lse - lse_ref).abs()
    assert float(d.max()) <= LSE_ABS, f"LSE {float(d.max()):.3e}"
    return float(err.max())


@pytest.mark.parametrize("cfg,max_seqs", [(2, 64), (3, 48), (5, 48)])
def test_decode_matches_fa4(cuda_device, fa4, cfg, max_seqs):
    batch = workloads.make_config(cfg, device=cuda_device, max_seqs=max_seqs)
    compare(fa4, batch)


def test_mixed_prefill_and_decode_match_fa4(cuda_device, fa4):
    """Config-4 shapes (32q/8kv): decode rows then chunked-prefill chunks on
    existing contexts, one varlen call for FA4."""
    q_lens = [1] * 12 + [2048, 300, 17, 1]
    ctx = [512, 8000, 1500, 3333, 700, 6000, 2048, 4097, 900, 1, 16, 7777] + [1900, 0, 4096, 129]
    seq_lens = [c + q for c, q in zip(ctx, q_lens)]
    # the decode-first order vLLM's reorder gives; the trailing 1-token row
    # belongs to the prefill group (it follows a chunk)
    batch = workloads.make_batch(q_lens, seq_lens, 32, 8, seed=41, device=cuda_device)
    compare(fa4, batch)


@pytest.mark.parametrize("hq,hkv,dtype", [(16, 16, torch.bfloat16), (64, 4, torch.bfloat16),
                                          (32, 8, torch.float16)])
def test_group_sizes_and_dtypes_match_fa4(cuda_device, fa4, hq, hkv, dtype):
    q_lens = [1] * 6 + [513, 64]
    seq_lens = [4000, 17, 1, 2048, 9000, 333] + [513 + 1000, 64 + 31]
    batch = workloads.make_batch(q_lens, seq_lens, hq, hkv, dtype=dtype, seed=hq + hkv,
                                 device=cuda_device)
    compare(fa4, batch)
