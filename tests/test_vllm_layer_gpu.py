"""GPU: the PS backend inside vLLM's own attention layer, as prime-rl's
inference server runs it (``vllm/model_executor/layers/attention/attention.py``
``Attention.forward`` -> ``torch.ops.vllm.unified_attention_with_output``,
``:437-530,691-761``), against vLLM's FLASH_ATTN backend (FA4 on sm_100) on
the same inputs.

A real ``VllmConfig`` is built from a Qwen3-0.6B-shaped ``config.json``
(16 query / 8 KV heads, head size 128; no weights are needed by an attention
layer).  The PS backend is registered as ``CUSTOM`` and picked by vLLM's own
backend selector (``attention_config.backend``); the FlashAttention layer is
vLLM's stock backend.  Each backend's metadata builder turns the same
``CommonAttentionMetadata`` into its metadata, and the layers run under
``set_forward_context`` exactly as the model runner calls them: eagerly on a
mixed decode + prefill batch, and for a decode batch from a CUDA graph
captured once and replayed over the next step's inputs (vLLM's full-graph
decode, ``AttentionCGSupport.UNIFORM_SINGLE_TOKEN_DECODE``).  Also covered:
``update_block_table`` and a layer that shares another layer's KV cache.
Bars: bf16 outputs within max-abs 2e-2 / mean-abs 2e-3 of FA4's, caches
bit-identical after the appends.
"""
from __future__ import annotations

import json

import pytest
import torch

from helpers import OUT_MAX_ABS, OUT_MEAN_ABS
from ps_attn import workloads

pytestmark = pytest.mark.gpu

HQ, HKV, D, BS = 16, 8, 128, 16
L_PS, L_FA, L_PS_SHARE, L_FA_SHARE = (f"model.layers.{i}.self_attn.attn" for i in range(4))
QWEN3_0_6B = {"architectures": ["Qwen3ForCausalLM"], "model_type": "qwen3", "hidden_size": 1024,
              "intermediate_size": 3072, "num_attention_heads": HQ, "num_key_value_heads": HKV,
              "head_dim": D, "num_hidden_layers": 4, "vocab_size": 151936, "max_position_embeddings": 40960,
              "rms_norm_eps": 1e-6, "rope_theta": 1000000, "torch_dtype": "bfloat16",
              "tie_word_embeddings": True, "attention_bias": False, "hidden_act": "silu"}


@pytest.fixture(scope="module")
def engine(cuda_device, tmp_path_factory):
    """vLLM config, the four attention layers (PS, FA, and one layer sharing
    each one's cache) and the two metadata builders."""
    pytest.importorskip("vllm")
    from vllm.config import CacheConfig, ModelConfig, VllmConfig, set_current_vllm_config
    from vllm.v1.attention.backends.flash_attn import FlashAttentionBackend
    from vllm.v1.attention.backends.registry import AttentionBackendEnum
    from vllm.v1.kv_cache_interface import FullAttentionSpec

    from vllm.model_executor.layers.attention.attention import Attention

    from ps_attn import backend as psb

    d = tmp_path_factory.mktemp("qwen3_0_6b_shapes")
    (d / "config.json").write_text(json.dumps(QWEN3_0_6B))
    mc = ModelConfig(model=str(d), skip_tokenizer_init=True, dtype="bfloat16", max_model_len=16384)
    vc = VllmConfig(model_config=mc, cache_config=CacheConfig(block_size=BS))
    psb.register()  # AttentionBackendEnum.CUSTOM -> the PS backend
    vc.attention_config.backend = AttentionBackendEnum.CUSTOM
    torch.set_default_dtype(torch.bfloat16)
    try:
        with set_current_vllm_config(vc):
            scale = D ** -0.5
            # the PS layer goes through vLLM's backend selector
            ps = Attention(HQ, D, scale, HKV, cache_config=vc.cache_config, prefix=L_PS)
            fa = Attention(HQ, D, scale, HKV, cache_config=vc.cache_config, prefix=L_FA,
                           attn_backend=FlashAttentionBackend)
            ps_share = Attention(HQ, D, scale, HKV, cache_config=vc.cache_config, prefix=L_PS_SHARE,
                                 kv_sharing_target_layer_name=L_PS)
            fa_share = Attention(HQ, D, scale, HKV, cache_config=vc.cache_config, prefix=L_FA_SHARE,
                                 kv_sharing_target_layer_name=L_FA, attn_backend=FlashAttentionBackend)
            spec = FullAttentionSpec(block_size=BS, num_kv_heads=HKV, head_size=D, dtype=torch.bfloat16)
            ps_builder = ps.attn_backend.get_builder_cls()(spec, [L_PS, L_PS_SHARE], vc, cuda_device)
            fa_builder = FlashAttentionBackend.get_builder_cls()(spec, [L_FA, L_FA_SHARE], vc, cuda_device)
    finally:
        torch.set_default_dtype(torch.float32)
    assert ps.attn_backend is psb.PSAttentionBackend, ps.attn_backend
    assert type(ps.impl).__name__ == "PSAttentionImpl"
    yield dict(vc=vc, ps=ps, fa=fa, ps_share=ps_share, fa_share=fa_share, ps_builder=ps_builder,
               fa_builder=fa_builder)


def common_metadata(batch):
    from vllm.v1.attention.backend import CommonAttentionMetadata

    qsl = batch.query_start_loc
    return CommonAttentionMetadata(
        query_start_loc=qsl, query_start_loc_cpu=qsl.cpu(), seq_lens=batch.seq_lens,
        num_reqs=batch.num_seqs, num_actual_tokens=batch.num_tokens, max_query_len=batch.max_query_len,
        max_seq_len=batch.max_seq_len, block_table_tensor=batch.block_table,
        slot_mapping=batch.slot_mapping, causal=True)


def bind(env, cache_ps, cache_fa):
    """Bind the caches as vLLM's bind_kv_cache does (a sharing layer gets its
    target's tensor)."""
    env["ps"].kv_cache = cache_ps
    env["ps_share"].kv_cache = cache_ps
    env["fa"].kv_cache = cache_fa
    env["fa_share"].kv_cache = cache_fa


def run_layers(env, cm, q, k, v, layers=("ps", "fa"), md=None):
    from vllm.forward_context import set_forward_context

    md_ps = env["ps_builder"].build(0, cm) if md is None else md
    md_fa = env["fa_builder"].build(0, cm)
    mds = {L_PS: md_ps, L_PS_SHARE: md_ps, L_FA: md_fa, L_FA_SHARE: md_fa}
    slots = {name: cm.slot_mapping for name in mds}
    outs = {}
    with set_forward_context(mds, env["vc"], slot_mapping=slots):
        for name in layers:
            outs[name] = env[name](q.flatten(1), k.flatten(1), v.flatten(1)).view(-1, HQ, D)
    return outs


def assert_close(a, b):
    err = (a.float() - b.float()).abs()
    assert torch.isfinite(a).all()
    assert float(err.max()) <= OUT_MAX_ABS, f"max abs {float(err.max()):.3e}"
    assert float(err.mean()) <= OUT_MEAN_ABS, f"mean abs {float(err.mean()):.3e}"


def test_mixed_batch_matches_flash_attention(cuda_device, engine):
    q_lens = [1] * 10 + [300, 17, 2048]
    ctx = [3000, 15, 1, 4096, 700, 1023, 1024, 1025, 2, 9000, 0, 4000, 333]
    batch = workloads.make_batch(q_lens, [c + q for c, q in zip(ctx, q_lens)], HQ, HKV, seed=7,
                                 device=cuda_device)
    cache_ps = batch.kv_cache.clone()
    cache_fa = batch.kv_cache.clone()
    bind(engine, cache_ps, cache_fa)
    cm = common_metadata(batch)
    outs = run_layers(engine, cm, batch.q, batch.key, batch.value)
    torch.cuda.synchronize()
    assert torch.equal(cache_ps.view(torch.int16), cache_fa.view(torch.int16))
    assert_close(outs["ps"], outs["fa"])
    # a layer reading the first layer's cache (KV sharing): no append of its own
    q2 = torch.randn_like(batch.q)
    outs2 = run_layers(engine, cm, q2, batch.key, batch.value, layers=("ps_share", "fa_share"))
    torch.cuda.synchronize()
    assert torch.equal(cache_ps.view(torch.int16), cache_fa.view(torch.int16))
    assert_close(outs2["ps_share"], outs2["fa_share"])


def test_update_block_table_relabels_pages(cuda_device, engine):
    """update_block_table (vLLM's hybrid allocator) with every page moved to
    another physical block gives the same output as the original table."""
    lens = [2049, 17, 4000, 1]
    batch = workloads.make_batch([1] * 4, lens, HQ, HKV, seed=9, device=cuda_device)
    cache = batch.kv_cache.clone()
    bind(engine, cache, batch.kv_cache.clone())
    cm = common_metadata(batch)
    md = engine["ps_builder"].build(0, cm)
    out_a = run_layers(engine, cm, batch.q, batch.key, batch.value, layers=("ps",), md=md)["ps"].clone()
    nb = cache.shape[1]
    perm = torch.randperm(nb, generator=torch.Generator().manual_seed(3)).to(cuda_device)
    moved = torch.empty_like(cache)
    moved[:, perm] = cache
    cache.copy_(moved)
    new_bt = perm[batch.block_table.long()].to(torch.int32)
    pos = batch.seq_lens.long() - 1
    new_slots = new_bt.long().gather(1, (pos // BS)[:, None])[:, 0] * BS + pos % BS
    md2 = engine["ps_builder"].update_block_table(md, new_bt, new_slots)
    assert md2.block_table is new_bt and md.block_table is batch.block_table
    out_b = run_layers(engine, cm, batch.q, batch.key, batch.value, layers=("ps",), md=md2)["ps"]
    torch.cuda.synchronize()
    assert torch.equal(out_a, out_b)


def test_full_cuda_graph_decode_replays_the_next_step(cuda_device, engine):
    """Decode captured once in a CUDA graph over persistent input buffers
    (as vLLM's full-graph decode does), replayed after the buffers are
    refilled with the next step's inputs, equals FA4 run eagerly on them."""
    from vllm.forward_context import set_forward_context
    from vllm.v1.attention.backend import AttentionCGSupport

    assert engine["ps_builder"]._cudagraph_support == AttentionCGSupport.UNIFORM_SINGLE_TOKEN_DECODE
    steps = 3
    lens = workloads.config_lengths(2)[1][:32]
    # pages for the last step's lengths; step 0 starts `steps` tokens earlier
    batch = workloads.make_batch([1] * 32, lens, HQ, HKV, seed=11, device=cuda_device)
    batch.seq_lens.sub_(steps)
    batch.max_seq_len -= steps
    pos = batch.seq_lens.long() - 1
    batch.slot_mapping.copy_(batch.block_table.long().gather(1, (pos // BS)[:, None])[:, 0] * BS + pos % BS)
    cache_ps = batch.kv_cache.clone()
    cache_fa = batch.kv_cache.clone()
    bind(engine, cache_ps, cache_fa)
    # persistent buffers of the captured step
    q, k, v = batch.q.clone(), batch.key.clone(), batch.value.clone()
    cm = common_metadata(batch)
    md = engine["ps_builder"].build(0, cm)
    mds = {L_PS: md}
    slots = {L_PS: cm.slot_mapping}
    stream = torch.cuda.Stream(cuda_device)
    with set_forward_context(mds, engine["vc"], slot_mapping=slots), torch.cuda.stream(stream):
        engine["ps"](q.flatten(1), k.flatten(1), v.flatten(1))  # warm-up (step 0)
        stream.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            out = engine["ps"](q.flatten(1), k.flatten(1), v.flatten(1)).view(-1, HQ, D)
    # the reference side runs step 0 too
    run_layers(engine, cm, batch.q, batch.key, batch.value, layers=("fa",))
    torch.cuda.synchronize()
    assert torch.equal(cache_ps.view(torch.int16), cache_fa.view(torch.int16))
    g_ = torch.Generator(device=cuda_device).manual_seed(12)
    for step in range(1, steps + 1):
        # next step: one more token per sequence, its slot, fresh q/k/v, all in place
        batch.seq_lens.add_(1)
        pos = batch.seq_lens.long() - 1
        batch.slot_mapping.copy_(batch.block_table.long().gather(1, (pos // BS)[:, None])[:, 0] * BS + pos % BS)
        batch.max_seq_len += 1
        for t in (q, k, v):
            t.copy_(torch.randn(t.shape, generator=g_, device=cuda_device, dtype=t.dtype))
        with torch.cuda.stream(stream):
            g.replay()
        stream.synchronize()
        cm_next = common_metadata(batch)
        ref = run_layers(engine, cm_next, q, k, v, layers=("fa",))["fa"]
        torch.cuda.synchronize()
        assert torch.equal(cache_ps.view(torch.int16), cache_fa.view(torch.int16)), step
        assert_close(out, ref)
    del g
