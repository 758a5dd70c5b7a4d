"""CPU: the vLLM backend surface (static API, metadata split, forward routing).

Kernels are replaced by recorders here; their numerics are covered by the GPU
tests.  vLLM's own ABCs and ``split_decodes_and_prefills`` are used as-is.
"""
from __future__ import annotations

import pytest
import torch

vllm_backend = pytest.importorskip("vllm.v1.attention.backend")

from ps_attn import _lib  # noqa: E402
from ps_attn import backend as psb  # noqa: E402


def test_static_api_matches_flash_attention_surface():
    from vllm.v1.attention.backends.flash_attn import FlashAttentionBackend

    B = psb.PSAttentionBackend
    for args in [(256, 16, 8, 128), (1000, 32, 1, 128), (7, 64, 4, 128)]:
        assert B.get_kv_cache_shape(*args) == FlashAttentionBackend.get_kv_cache_shape(*args)
    with pytest.raises(ValueError):
        B.get_kv_cache_shape(10, 24, 8, 128)
    assert B.get_kv_cache_stride_order() == (0, 1, 2, 3, 4)
    # the append runs inside forward (decode tokens fused into the decode launch)
    assert B.forward_includes_kv_cache_update is True
    assert B.get_impl_cls() is psb.PSAttentionImpl
    assert B.get_builder_cls() is psb.PSAttentionMetadataBuilder
    assert B.supports_head_size(128) and not B.supports_head_size(64)
    assert torch.bfloat16 in B.supported_dtypes and torch.float16 in B.supported_dtypes
    assert B.get_name() == "CUSTOM"


def test_registration_overrides_registry():
    from vllm.v1.attention.backends.registry import AttentionBackendEnum

    psb.register()
    assert AttentionBackendEnum.CUSTOM.get_class() is psb.PSAttentionBackend
    AttentionBackendEnum.CUSTOM.clear_override()


@pytest.mark.parametrize("kw", [dict(alibi_slopes=[1.0]), dict(sliding_window=128),
                                dict(logits_soft_cap=30.0), dict(kv_cache_dtype="fp8_e5m2")])
def test_impl_rejects_unsupported_options(kw):
    base = dict(num_heads=16, head_size=128, scale=0.088, num_kv_heads=8, alibi_slopes=None,
                sliding_window=None, kv_cache_dtype="auto")
    base.update(kw)
    with pytest.raises(NotImplementedError):
        psb.PSAttentionImpl(**base)


def _common(q_lens, seq_lens):
    from vllm.v1.attention.backend import CommonAttentionMetadata

    qsl = torch.zeros(len(q_lens) + 1, dtype=torch.int32)
    qsl[1:] = torch.cumsum(torch.tensor(q_lens), 0)
    T = int(qsl[-1])
    return CommonAttentionMetadata(
        query_start_loc=qsl, query_start_loc_cpu=qsl.clone(),
        seq_lens=torch.tensor(seq_lens, dtype=torch.int32), num_reqs=len(q_lens),
        num_actual_tokens=T, max_query_len=max(q_lens), max_seq_len=max(seq_lens),
        block_table_tensor=torch.zeros(len(q_lens), 8, dtype=torch.int32),
        slot_mapping=torch.arange(T, dtype=torch.int64))


def _builder():
    b = psb.PSAttentionMetadataBuilder.__new__(psb.PSAttentionMetadataBuilder)
    b.workspace = object()
    return b


def test_builder_splits_decode_first_batches():
    md = _builder().build(0, _common([1, 1, 1, 7, 30], [10, 20, 30, 40, 90]))
    assert (md.num_decodes, md.num_decode_tokens, md.num_prefills) == (3, 3, 2)
    md = _builder().build(0, _common([1, 1], [5, 6]))
    assert (md.num_decodes, md.num_prefills) == (2, 0)
    with pytest.raises(NotImplementedError):
        _builder().build(16, _common([1, 1], [5, 6]))


def test_forward_routes_decode_and_prefill(monkeypatch):
    calls = []
    monkeypatch.setattr(psb.ops, "paged_decode", lambda *a, **k: calls.append(("decode", a, k)))
    monkeypatch.setattr(psb.ops, "chunked_prefill", lambda *a, **k: calls.append(("prefill", a, k)))
    impl = psb.PSAttentionImpl(16, 128, 0.088, 8, None, None, "auto")
    md = _builder().build(0, _common([1, 1, 5], [10, 20, 40]))
    T = 7
    q = torch.zeros(T + 2, 16, 128)  # padded rows beyond num_actual_tokens
    out = torch.zeros(T + 2, 16, 128)
    kv = torch.zeros(2, 4, 16, 8, 128)
    impl.forward(None, q, None, None, kv, md, out)
    assert [c[0] for c in calls] == ["decode", "prefill"]
    _, a, k = calls[0]
    assert a[0].shape[0] == 2 and a[3].shape[0] == 2 and a[4].tolist() == [10, 20]
    assert k["query_start_loc"].tolist() == [0, 1, 2]
    _, a, k = calls[1]
    assert a[0].shape[0] == T and a[3].shape[0] == 1 and a[4].tolist() == [40]
    assert a[5].tolist() == [2, 7]
    # profiling run: zero output, no kernels
    calls.clear()
    out.fill_(3)
    impl.forward(None, q, None, None, kv, None, out)
    assert calls == [] and not out.any()


def test_forward_appends_prefill_tokens_and_fuses_decode(monkeypatch):
    calls = []
    monkeypatch.setattr(psb.ops, "kv_append", lambda *a, **k: calls.append(("append", a, k)))
    monkeypatch.setattr(psb.ops, "paged_decode", lambda *a, **k: calls.append(("decode", a, k)))
    monkeypatch.setattr(psb.ops, "chunked_prefill", lambda *a, **k: calls.append(("prefill", a, k)))
    impl = psb.PSAttentionImpl(16, 128, 0.088, 8, None, None, "auto")
    md = _builder().build(0, _common([1, 1, 5], [10, 20, 40]))
    T = 7
    q = torch.zeros(T + 1, 16, 128)
    key = torch.randn(T + 1, 8, 128)
    val = torch.randn(T + 1, 8, 128)
    out = torch.zeros(T + 1, 16, 128)
    impl.forward(None, q, key, val, torch.zeros(2, 4, 16, 8, 128), md, out)
    assert [c[0] for c in calls] == ["append", "decode", "prefill"]
    _, a, _ = calls[0]
    assert a[0].shape[0] == 5 and a[4].tolist() == [2, 3, 4, 5, 6]  # prefill rows only
    _, _, k = calls[1]
    assert k["new_key"] is key and k["slot_mapping"] is md.slot_mapping


def test_kv_update_unbinds_cache(monkeypatch):
    seen = {}
    monkeypatch.setattr(psb.ops, "kv_append",
                        lambda k, v, kc, vc, s: seen.update(kc=kc, vc=vc, s=s))
    impl = psb.PSAttentionImpl(16, 128, 0.088, 8, None, None, "auto")
    kv = torch.zeros(2, 4, 16, 8, 128)
    impl.do_kv_cache_update(None, torch.zeros(3, 8, 128), torch.zeros(3, 8, 128), kv,
                            torch.arange(3))
    assert seen["kc"].data_ptr() == kv[0].data_ptr() and seen["vc"].data_ptr() == kv[1].data_ptr()


def test_cascade_opt_in_builds_one_plan_per_step(monkeypatch):
    """With PS_ATTN_CASCADE=1 the builder builds the shared-prefix plan for the
    decode rows (the same slices forward() passes) and forward hands it on."""
    built, calls = [], []
    monkeypatch.setattr(psb.ops, "cascade_plan",
                        lambda bt, sl, hq, hkv, bs, query_start_loc=None, plan=None:
                        built.append((bt.shape[0], sl.tolist(), query_start_loc.tolist(), bs)) or "PLAN")
    monkeypatch.setattr(psb.ops, "paged_decode", lambda *a, **k: calls.append(k))
    monkeypatch.setattr(psb.ops, "chunked_prefill", lambda *a, **k: None)
    b = _builder()
    b.cascade, b.plan, b.block_size = True, None, 16
    b.num_heads_q, b.num_heads_kv = 16, 8
    md = b.build(0, _common([1, 1, 1, 7], [10, 20, 30, 40]))
    assert built == [(3, [10, 20, 30], [0, 1, 2, 3], 16)] and md.cascade_plan == "PLAN"
    impl = psb.PSAttentionImpl(16, 128, 0.088, 8, None, None, "auto")
    impl.forward(None, torch.zeros(10, 16, 128), None, None, torch.zeros(2, 4, 16, 8, 128), md,
                 torch.zeros(10, 16, 128))
    assert calls[0]["cascade"] == "PLAN"
    # off by default
    monkeypatch.delenv("PS_ATTN_CASCADE", raising=False)
    assert not psb.cascade_enabled()
    monkeypatch.setenv("PS_ATTN_CASCADE", "1")
    assert psb.cascade_enabled()


def test_rope_fusion_variant(monkeypatch):
    """The rope_fusion variant: vLLM issues the KV update (the backend says
    forward does not include it), the fused RoPE hook unbinds the cache and
    calls ps_rope_kv_append, and forward does not append."""
    from vllm.v1.attention.backends.registry import AttentionBackendEnum

    B = psb.PSRopeAttentionBackend
    assert B.forward_includes_kv_cache_update is False and B.get_impl_cls() is psb.PSRopeAttentionImpl
    psb.register(rope_fusion=True)
    assert AttentionBackendEnum.CUSTOM.get_class() is B
    AttentionBackendEnum.CUSTOM.clear_override()
    seen, calls = {}, []
    monkeypatch.setattr(psb.ops, "rope_kv_append", lambda *a: seen.update(args=a))
    monkeypatch.setattr(psb.ops, "kv_append", lambda *a, **k: calls.append("append"))
    monkeypatch.setattr(psb.ops, "paged_decode", lambda *a, **k: calls.append(("decode", k)))
    monkeypatch.setattr(psb.ops, "chunked_prefill", lambda *a, **k: calls.append("prefill"))
    impl = psb.PSRopeAttentionImpl(16, 128, 0.088, 8, None, None, "auto")
    assert impl.fused_rope_kvcache_supported()
    kv = torch.zeros(2, 4, 16, 8, 128)
    q, k, v = torch.zeros(3, 16 * 128), torch.zeros(3, 8 * 128), torch.zeros(3, 8 * 128)
    pos, cs, slots = torch.arange(3).view(1, 3), torch.zeros(10, 128), torch.arange(3)
    impl.do_rope_and_kv_cache_update(None, q, k, v, pos, cs, True, kv, slots)
    a = seen["args"]
    assert a[0] is q and a[1] is k and a[3].shape == (3,) and a[5] is True
    assert a[6].data_ptr() == kv[0].data_ptr() and a[7].data_ptr() == kv[1].data_ptr()
    md = _builder().build(0, _common([1, 1, 5], [10, 20, 40]))
    impl.forward(None, torch.zeros(8, 16, 128), torch.zeros(8, 8, 128), torch.zeros(8, 8, 128),
                 kv, md, torch.zeros(8, 16, 128))
    assert calls[0][0] == "decode" and "new_key" not in calls[0][1] and calls[1] == "prefill"


def test_fp8_cache_routes_scales_and_dequantized_prefill(monkeypatch):
    calls = []
    monkeypatch.setattr(psb.ops, "kv_append", lambda *a, **k: calls.append(("append", a, k)))
    monkeypatch.setattr(psb.ops, "paged_decode", lambda *a, **k: calls.append(("decode", a, k)))
    monkeypatch.setattr(psb.ops, "chunked_prefill", lambda *a, **k: calls.append(("prefill", a, k)))

    def fake_gather(kc, vc, bt, sl, max_pages, dtype, **k):
        calls.append(("gather", (bt, sl, max_pages, dtype), k))
        return "kd", "vd", "bt"

    monkeypatch.setattr(psb.ops, "dequant_gather", fake_gather)
    assert "fp8" in psb.PSAttentionBackend.supported_kv_cache_dtypes
    impl = psb.PSAttentionImpl(16, 128, 0.088, 8, None, None, "fp8")

    class Layer:
        _k_scale = torch.tensor(0.5)
        _v_scale = torch.tensor(0.25)

    md = _builder().build(0, _common([1, 1, 5], [10, 20, 40]))
    T = 7
    q = torch.zeros(T, 16, 128, dtype=torch.bfloat16)
    kv = torch.zeros(2, 4, 16, 8, 128, dtype=torch.uint8)
    impl.forward(Layer(), q, torch.zeros(T, 8, 128), torch.zeros(T, 8, 128), kv, md,
                 torch.zeros(T, 16, 128, dtype=torch.bfloat16))
    assert [c[0] for c in calls] == ["append", "decode", "gather", "prefill"]
    for name, _, k in calls:
        if name in ("append", "decode", "prefill"):
            assert k["k_scale"] is Layer._k_scale and k["v_scale"] is Layer._v_scale
    assert "k_scale" not in calls[2][2]  # the scratch holds the unscaled e4m3 values
    _, (bt, sl, max_pages, dtype), _ = calls[2]
    assert max_pages == 3 and sl.tolist() == [40] and dtype == torch.bfloat16  # ceil(40 / 16)
    _, a, _ = calls[3]
    assert a[1] == "kd" and a[2] == "vd" and a[3] == "bt"


def test_forward_routes_dcp_batches(monkeypatch):
    """Under decode context parallelism (vLLM's DCP group of 2) decode rows go
    to dcp.dcp_decode and prefill chunks to dcp.dcp_prefill, with the chunk
    offsets rebased to the first prefill row; fp8 caches are refused."""
    import vllm.distributed.parallel_state as ps_state

    from ps_attn import dcp

    class Group:
        world_size, rank_in_group = 2, 0

    monkeypatch.setattr(ps_state, "get_dcp_group", lambda: Group())
    with pytest.raises(NotImplementedError, match="fp8"):
        psb.PSAttentionImpl(16, 128, 0.088, 8, None, None, "fp8")
    impl = psb.PSAttentionImpl(16, 128, 0.088, 8, None, None, "auto")
    calls = []
    monkeypatch.setattr(dcp, "dcp_decode", lambda *a, **k: calls.append(("decode", a, k)))
    monkeypatch.setattr(dcp, "dcp_prefill", lambda *a, **k: calls.append(("prefill", a, k)))
    md = _builder().build(0, _common([1, 1, 5, 3], [10, 20, 40, 9]))
    md.dcp_comm = "comm"
    T = 10
    q = torch.zeros(T, 16, 128)
    key, val = torch.randn(T, 8, 128), torch.randn(T, 8, 128)
    out = torch.zeros(T, 16, 128)
    impl.forward(None, q, key, val, torch.zeros(2, 4, 16, 8, 128), md, out)
    assert [c[0] for c in calls] == ["decode", "prefill"]
    _, a, _ = calls[0]
    assert a[0] == "comm" and a[1].shape[0] == 2 and a[5].tolist() == [10, 20] and a[8].shape[0] == 2
    _, a, _ = calls[1]
    assert a[1].shape[0] == 8 and a[5].tolist() == [40, 9] and a[6].tolist() == [0, 5, 8]
    assert a[7] == 5 and a[10].shape[0] == 8 and a[12].tolist() == list(range(2, 10))


def test_rope_fusion_variant_declines_fp8_cache():
    impl = psb.PSRopeAttentionImpl(16, 128, 0.088, 8, None, None, "fp8")
    assert impl.fused_rope_kvcache_supported() is False
    assert psb.PSRopeAttentionImpl(16, 128, 0.088, 8, None, None, "auto").fused_rope_kvcache_supported()


def test_builder_sets_up_the_dcp_group(monkeypatch):
    """With decode_context_parallel_size > 1 the metadata builder maps the
    group's slabs once (over the DCP group's CPU process group), sizes the
    rows for a whole prefill step and hands the group to every metadata."""
    from types import SimpleNamespace

    import vllm.distributed.parallel_state as ps_state

    from ps_attn import dcp

    seen = {}

    class Comm:
        def workspace(self, rows, hkv, head_size):
            seen["ws"] = (rows, hkv, head_size)
            return "ws"

    def fake_from_pg(rows, hq_local, interleave, group=None, device=None):
        seen.update(rows=rows, hq_local=hq_local, interleave=interleave, group=group)
        return Comm()

    monkeypatch.setattr(ps_state, "get_dcp_group", lambda: SimpleNamespace(cpu_group="cpu-group"))
    monkeypatch.setattr(dcp.DcpComm, "from_process_group", staticmethod(fake_from_pg))
    mc = SimpleNamespace(get_num_attention_heads=lambda pc: 16, get_num_kv_heads=lambda pc: 8,
                         get_head_size=lambda: 128)
    pc = SimpleNamespace(decode_context_parallel_size=2, cp_kv_cache_interleave_size=4)
    cfg = SimpleNamespace(model_config=mc, parallel_config=pc,
                          scheduler_config=SimpleNamespace(max_num_seqs=64, max_num_batched_tokens=8192),
                          compilation_config=SimpleNamespace(max_cudagraph_capture_size=128))
    b = psb.PSAttentionMetadataBuilder(SimpleNamespace(block_size=16), ["l0"], cfg, torch.device("cpu"))
    # rows capped at what one ps_dcp_decode call takes (larger steps run in pieces)
    assert seen["rows"] == _lib.PS_DCP_MAX_TOKENS == 4096
    assert seen["hq_local"] == 16 and seen["interleave"] == 4
    assert seen["group"] == "cpu-group" and seen["ws"] == (4096, 8, 128)
    lib = _lib.load()  # the library accepts the capped rows, and nothing above
    assert lib.ps_dcp_slab_bytes(seen["rows"], 16, 2) > 0
    assert lib.ps_dcp_slab_bytes(seen["rows"] + 1, 16, 2) == -1
    md = b.build(0, _common([1, 3], [10, 20]))
    assert isinstance(md.dcp_comm, Comm) and md.workspace == "ws" and md.cascade_plan is None
