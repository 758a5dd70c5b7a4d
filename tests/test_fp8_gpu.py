"""GPU: fp8 (e4m3) KV cache -- the append bit-exact against the oracle (and
against vLLM's compiled reshape_and_cache_flash with kv_cache_dtype "fp8"
where it loads), and the decode against fp32 attention over the dequantized
cache (code * scale), with the attention tolerances."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import assert_attn_close, to_np32
from oracle import ps_oracle
from ps_attn import _lib, ops, workloads

pytestmark = pytest.mark.gpu


def _scales(dev, ks=0.037, vs=0.021):
    return (torch.tensor(ks, dtype=torch.float32, device=dev),
            torch.tensor(vs, dtype=torch.float32, device=dev))


def _fp8_batch(q_lens, seq_lens, hq, hkv, dtype, seed, block_size=16, stale_nan=True, gain=2.0):
    """A batch whose cache is fp8: the cached tokens are e4m3 codes of
    gain * N(0,1) / scale data; unused rows hold random codes, NaN codes
    included."""
    b = workloads.make_batch(q_lens, seq_lens, hq, hkv, dtype=dtype, seed=seed, block_size=block_size)
    g = torch.Generator().manual_seed(seed + 5)
    codes = torch.randint(0, 256, tuple(b.kv_cache.shape), generator=g, dtype=torch.uint8)
    if not stale_nan:
        codes[(codes & 0x7F) == 0x7F] = 0
    ks, vs = 0.037, 0.021
    # cached tokens of every sequence: quantized N(0,1) values
    real = ps_oracle.e4m3_encode(b.kv_cache.float().numpy() * np.float32(gain) /
                                 np.array([ks, vs], np.float32)[:, None, None, None, None])
    bt, L = b.block_table.numpy(), b.seq_lens.numpy()
    mask = np.zeros(tuple(b.kv_cache.shape[1:3]), bool)
    for i, n in enumerate(L):
        for pos in range(n):
            mask[bt[i, pos // block_size], pos % block_size] = True
    codes_np = codes.numpy()
    codes_np[:, mask] = real[:, mask]
    return b, torch.from_numpy(codes_np), ks, vs


def _oracle_decode(b, codes, ks, vs):
    kc = ps_oracle.dequantize_cache(codes[0].numpy(), ks)
    vc = ps_oracle.dequantize_cache(codes[1].numpy(), vs)
    return ps_oracle.paged_attention(to_np32(b.q), kc, vc, b.block_table.numpy(), b.seq_lens.numpy(),
                                     b.query_start_loc.numpy(), b.softmax_scale)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_fp8_append_bit_exact(cuda_device, dtype):
    g = torch.Generator().manual_seed(11)
    T, H, D, NB, bs = 37, 8, 128, 9, 16
    # key/value as views of a wider qkv row, like vLLM's
    qkv = (torch.randn(T, (4 + 2 * H) * D, generator=g) * 9).to(dtype)
    qkv[0, 4 * D] = 1e4  # saturates to 448
    key = qkv[:, 4 * D:(4 + H) * D].view(T, H, D)
    value = qkv[:, (4 + H) * D:].view(T, H, D)
    kc = torch.randint(0, 256, (NB, bs, H, D), generator=g, dtype=torch.uint8)
    vc = torch.randint(0, 256, (NB, bs, H, D), generator=g, dtype=torch.uint8)
    slots = torch.randperm(NB * bs, generator=g)[:T].to(torch.int64)
    slots[3] = -1
    kc_ref, vc_ref = kc.numpy().copy(), vc.numpy().copy()
    ps_oracle.kv_append_fp8(key.float().numpy(), value.float().numpy(), kc_ref, vc_ref, slots.numpy(),
                            0.37, 1.7)
    kd, vd, sd = kc.to(cuda_device), vc.to(cuda_device), slots.to(cuda_device)
    ks, vs = _scales(cuda_device, 0.37, 1.7)
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    ops.kv_append(key.to(cuda_device), value.to(cuda_device), kd, vd, sd, status=status,
                  k_scale=ks, v_scale=vs)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert np.array_equal(kd.cpu().numpy(), kc_ref) and np.array_equal(vd.cpu().numpy(), vc_ref)
    assert ps_oracle.e4m3_decode(kc_ref.reshape(-1)[:1]).shape == (1,)
    # float8_e4m3fn-typed caches take the same path
    k8 = kc.to(cuda_device).view(torch.float8_e4m3fn)
    v8 = vc.to(cuda_device).view(torch.float8_e4m3fn)
    ops.kv_append(key.to(cuda_device), value.to(cuda_device), k8, v8, sd, k_scale=ks, v_scale=vs)
    torch.cuda.synchronize()
    assert np.array_equal(k8.view(torch.uint8).cpu().numpy(), kc_ref)


def test_fp8_append_matches_vllm_compiled_op(cuda_device):
    try:
        from vllm import _custom_ops as vops  # noqa: F401
        fn = torch.ops._C_cache_ops.reshape_and_cache_flash
    except Exception as e:  # pragma: no cover - depends on the box's vLLM build
        pytest.skip(f"vLLM compiled cache ops unavailable: {e}")
    g = torch.Generator().manual_seed(12)
    T, H, D, NB, bs = 64, 8, 128, 8, 16
    key = (torch.randn(T, H, D, generator=g) * 5).to(torch.bfloat16).to(cuda_device)
    value = (torch.randn(T, H, D, generator=g) * 5).to(torch.bfloat16).to(cuda_device)
    slots = torch.randperm(NB * bs, generator=g)[:T].to(torch.int64).to(cuda_device)
    ks, vs = _scales(cuda_device, 0.0173, 0.41)
    k1 = torch.zeros(NB, bs, H, D, dtype=torch.uint8, device=cuda_device)
    v1 = torch.zeros_like(k1)
    k2, v2 = k1.clone(), v1.clone()
    fn(key, value, k1, v1, slots, "fp8", ks, vs)
    ops.kv_append(key, value, k2, v2, slots, k_scale=ks, v_scale=vs)
    torch.cuda.synchronize()
    nk = int((k1 != k2).sum())
    nv = int((v1 != v2).sum())
    assert nk == 0 and nv == 0, f"{nk} key and {nv} value codes differ from vLLM's op"


@pytest.mark.parametrize("group", [1, 2, 4, 8, 16])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_fp8_decode_matches_dequantized_attention(cuda_device, group, dtype):
    hkv = 2
    lens = [1, 15, 16, 17, 333, 2049, 40]
    b, codes, ks, vs = _fp8_batch([1] * len(lens), lens, group * hkv, hkv, dtype, seed=300 + group)
    rout, rlse = _oracle_decode(b, codes, ks, vs)
    g = b.to(cuda_device)
    kc, vc = codes[0].to(cuda_device), codes[1].to(cuda_device)
    kss, vss = _scales(cuda_device, ks, vs)
    out = torch.full_like(g.q, float("nan"))
    lse = torch.empty(g.q.shape[1], g.q.shape[0], dtype=torch.float32, device=cuda_device)
    ws = ops.DecodeWorkspace(len(lens), group * hkv, hkv, 128, cuda_device)
    ops.paged_decode(g.q, kc, vc, g.block_table, g.seq_lens, g.softmax_scale, out, lse=lse,
                     query_start_loc=g.query_start_loc, workspace=ws, k_scale=kss, v_scale=vss)
    torch.cuda.synchronize()
    assert ws.status() == 0
    assert_attn_close(to_np32(out), rout, to_np32(lse), rlse)


@pytest.mark.parametrize("block_size", [16, 32])
def test_fp8_decode_fused_append_and_block_sizes(cuda_device, block_size):
    """The new token is quantized into the cache inside the decode launch and
    attended to: same cache bytes as ps_kv_append_fp8, same output as the
    oracle over the updated, dequantized cache."""
    lens = [3, 64, 65, 500, 1200]
    b, codes, ks, vs = _fp8_batch([1] * len(lens), lens, 32, 8, torch.bfloat16, seed=41,
                                  block_size=block_size, stale_nan=False)
    kc_ref, vc_ref = codes[0].numpy().copy(), codes[1].numpy().copy()
    ps_oracle.kv_append_fp8(to_np32(b.key), to_np32(b.value), kc_ref, vc_ref, b.slot_mapping.numpy(), ks, vs)
    rout, rlse = ps_oracle.paged_attention(
        to_np32(b.q), ps_oracle.dequantize_cache(kc_ref, ks), ps_oracle.dequantize_cache(vc_ref, vs),
        b.block_table.numpy(), b.seq_lens.numpy(), b.query_start_loc.numpy(), b.softmax_scale)
    g = b.to(cuda_device)
    kc, vc = codes[0].to(cuda_device), codes[1].to(cuda_device)
    kss, vss = _scales(cuda_device, ks, vs)
    out = torch.empty_like(g.q)
    lse = torch.empty(g.q.shape[1], g.q.shape[0], dtype=torch.float32, device=cuda_device)
    ws = ops.DecodeWorkspace(len(lens), 32, 8, 128, cuda_device)
    ops.paged_decode(g.q, kc, vc, g.block_table, g.seq_lens, g.softmax_scale, out, lse=lse,
                     query_start_loc=g.query_start_loc, workspace=ws, new_key=g.key, new_value=g.value,
                     slot_mapping=g.slot_mapping, k_scale=kss, v_scale=vss)
    torch.cuda.synchronize()
    assert ws.status() == 0
    assert np.array_equal(kc.cpu().numpy(), kc_ref) and np.array_equal(vc.cpu().numpy(), vc_ref)
    assert_attn_close(to_np32(out), rout, to_np32(lse), rlse)


def test_fp8_cache_refused_where_not_built(cuda_device):
    b = workloads.make_batch([4], [40], 16, 8, seed=2).to(cuda_device)
    kc = torch.zeros(b.kv_cache.shape[1:], dtype=torch.uint8, device=cuda_device)
    out = torch.empty_like(b.q)
    with pytest.raises(_lib.PSError) as e:
        ops.chunked_prefill(b.q, kc, kc.clone(), b.block_table, b.seq_lens, b.query_start_loc,
                            b.softmax_scale, out)
    assert e.value.code == _lib.PS_ERR_UNSUPPORTED


def test_dequant_gather_matches_oracle(cuda_device):
    """Pages each sequence covers, dequantized to bf16 (code * scale rounded
    once), at the compact block table's positions."""
    g = torch.Generator().manual_seed(21)
    NB, bs, H, D = 40, 16, 4, 128
    codes = torch.randint(0, 256, (2, NB, bs, H, D), generator=g, dtype=torch.uint8)
    codes[(codes & 0x7F) == 0x7F] = 1  # no NaN codes in covered pages
    lens = torch.tensor([1, 16, 17, 100, 0], dtype=torch.int32)
    maxp = 8
    bt = torch.randperm(NB, generator=g)[:5 * maxp].to(torch.int32).view(5, maxp)
    ks, vs = _scales(cuda_device, 0.75, 1.5)
    kd, vd, cbt = ops.dequant_gather(codes[0].to(cuda_device), codes[1].to(cuda_device),
                                     bt.to(cuda_device), lens.to(cuda_device), maxp, torch.bfloat16,
                                     k_scale=ks, v_scale=vs)
    torch.cuda.synchronize()
    assert torch.equal(cbt.cpu(), torch.arange(5 * maxp, dtype=torch.int32).view(5, maxp))
    for b, L in enumerate(lens.tolist()):
        for p in range((L + bs - 1) // bs):
            for src, dst, s in ((codes[0], kd, 0.75), (codes[1], vd, 1.5)):
                want = ps_oracle.round_to(ps_oracle.dequantize_cache(src[bt[b, p]].numpy(), s), "bf16")
                assert np.array_equal(dst[b * maxp + p].float().cpu().numpy(), want)


def test_backend_forward_over_fp8_cache(cuda_device):
    """vLLM backend with kv_cache_dtype "fp8": a decode-first mixed batch
    appends (quantized), decodes (fp8 kernel) and prefills (the e4m3 pages
    copied to bf16, scales in the kernel) -- attention over the updated,
    dequantized cache, N(0,1)-scale data as the attention tolerances assume."""
    pytest.importorskip("vllm.v1.attention.backend")
    from ps_attn import backend as psb

    q_lens, lens = [1, 1, 1, 37, 200], [40, 300, 17, 1025, 700]
    b, codes, ks, vs = _fp8_batch(q_lens, lens, 32, 8, torch.bfloat16, seed=61, stale_nan=False, gain=1.0)
    kc_ref, vc_ref = codes[0].numpy().copy(), codes[1].numpy().copy()
    ps_oracle.kv_append_fp8(to_np32(b.key), to_np32(b.value), kc_ref, vc_ref, b.slot_mapping.numpy(), ks, vs)
    rout, _ = ps_oracle.paged_attention(
        to_np32(b.q), ps_oracle.dequantize_cache(kc_ref, ks), ps_oracle.dequantize_cache(vc_ref, vs),
        b.block_table.numpy(), b.seq_lens.numpy(), b.query_start_loc.numpy(), b.softmax_scale)
    g = b.to(cuda_device)
    kv = codes.to(cuda_device)
    impl = psb.PSAttentionImpl(32, 128, g.softmax_scale, 8, None, None, "fp8")

    class Layer:
        _k_scale, _v_scale = _scales(cuda_device, ks, vs)

    T = g.q.shape[0]
    ws = ops.DecodeWorkspace(len(lens), 32, 8, 128, cuda_device)
    md = psb.PSAttentionMetadata(
        num_actual_tokens=T, max_query_len=max(q_lens), query_start_loc=g.query_start_loc,
        max_seq_len=max(lens), seq_lens=g.seq_lens, block_table=g.block_table,
        slot_mapping=g.slot_mapping, num_decodes=3, num_decode_tokens=3, num_prefills=2, workspace=ws)
    out = torch.full_like(g.q, float("nan"))
    impl.forward(Layer(), g.q, g.key, g.value, kv, md, out)
    torch.cuda.synchronize()
    assert ws.status() == 0
    assert np.array_equal(kv[0].cpu().numpy(), kc_ref) and np.array_equal(kv[1].cpu().numpy(), vc_ref)
    assert_attn_close(to_np32(out), rout)
