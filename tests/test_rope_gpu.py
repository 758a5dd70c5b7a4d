"""GPU: fused rotary embedding + KV append, bit-exact against vLLM's own
torch-native RoPE (golden vectors) and the oracle (RoPE restatement followed
by the append contract)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import GOLDEN, golden_meta
from oracle import ps_oracle
from ps_attn import _lib, ops

pytestmark = pytest.mark.gpu

CASES = sorted(golden_meta()["rope"])


def bits_to_tensor(a, dtype):
    if dtype == torch.bfloat16:
        return torch.from_numpy(a.astype(np.int16)).view(torch.bfloat16)
    return torch.from_numpy(a).to(dtype)


def tensor_to_f32(t):
    return t.detach().to("cpu", torch.float32).numpy()


@pytest.mark.parametrize("name", CASES)
def test_rope_append_matches_reference_golden(cuda_device, name):
    m = golden_meta()["rope"][name]
    d = dict(np.load(GOLDEN / f"rope_{name}.npz"))
    T, Hq, Hkv, D, rot, neox = (int(v) for v in d["shape"])
    dtype = torch.bfloat16 if "bfloat16" in m["dtype"] else torch.float16
    cdtype = {"torch.bfloat16": torch.bfloat16, "torch.float16": torch.float16,
              "torch.float32": torch.float32}[m["cache_dtype"]]
    pos = torch.from_numpy(d["positions"])
    cache = torch.zeros(m["max_position"], rot, dtype=cdtype)
    cache[pos] = bits_to_tensor(d["cos_sin_rows"], cdtype) if cdtype != torch.float32 \
        else torch.from_numpy(d["cos_sin_rows"])
    q = bits_to_tensor(d["q_in"], dtype).to(cuda_device)
    k = bits_to_tensor(d["k_in"], dtype).to(cuda_device)
    v = torch.randn(T, Hkv * D, dtype=dtype, device=cuda_device)
    NB, bs = 4, 16
    kc = torch.zeros(NB, bs, Hkv, D, dtype=dtype, device=cuda_device)
    vc = torch.zeros_like(kc)
    slots = torch.tensor([5, -1, 0, 63, 17, 18, 40, -1, 33], dtype=torch.int64, device=cuda_device)
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    ops.rope_kv_append(q, k, v, pos.to(cuda_device), cache.to(cuda_device), bool(neox), kc, vc,
                       slots, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    qo = bits_to_tensor(d["q_out"], dtype)
    ko = bits_to_tensor(d["k_out"], dtype)
    assert torch.equal(q.cpu(), qo) and torch.equal(k.cpu(), ko)
    # cache rows: the rotated key and the value at each non-negative slot
    ko3, v3 = ko.view(T, Hkv, D), v.cpu().view(T, Hkv, D)
    for t, s in enumerate(slots.tolist()):
        if s >= 0:
            assert torch.equal(kc.cpu()[s // bs, s % bs], ko3[t])
            assert torch.equal(vc.cpu()[s // bs, s % bs], v3[t])


@pytest.mark.parametrize("layout", ["aligned", "rot40", "offset"])
@pytest.mark.parametrize("neox", [True, False])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_rope_append_on_qkv_views_matches_oracle(cuda_device, neox, dtype, layout):
    """q, k, v as views of one fused qkv projection output (vLLM's layout),
    Qwen3-4B heads, a padding slot, fp32 cos/sin cache.  "aligned" takes the
    16-byte path; a rotary dim of 40 and rows that start 2 bytes off a 16-byte
    boundary take the element path."""
    g = torch.Generator(device=cuda_device).manual_seed(7)
    T, Hq, Hkv, D = 300, 32, 8, 128
    rot = 40 if layout == "rot40" else 128
    pad = 1 if layout == "offset" else 0
    qkv = torch.randn(T, (Hq + 2 * Hkv) * D + pad, generator=g, device=cuda_device).to(dtype)
    q, k, v = qkv[:, pad:].split([Hq * D, Hkv * D, Hkv * D], dim=-1)
    maxpos = 8192
    inv = 1.0 / (1e6 ** (torch.arange(0, rot, 2, dtype=torch.float32) / rot))
    f = torch.outer(torch.arange(maxpos, dtype=torch.float32), inv)
    cache = torch.cat((f.cos(), f.sin()), -1).to(cuda_device)
    pos = torch.randint(0, maxpos, (T,), generator=g, device=cuda_device)
    NB, bs = 40, 16
    kc = torch.randn(NB, bs, Hkv, D, generator=g, device=cuda_device).to(dtype)
    vc = torch.randn(NB, bs, Hkv, D, generator=g, device=cuda_device).to(dtype)
    slots = torch.randperm(NB * bs, generator=g, device=cuda_device)[:T].to(torch.int64)
    slots[11] = -1
    q0, k0, v0 = q.clone(), k.clone(), v.clone()
    kc0, vc0 = kc.clone(), vc.clone()
    ops.rope_kv_append(q, k, v, pos, cache, neox, kc, vc, slots)
    torch.cuda.synchronize()
    dt = "bf16" if dtype == torch.bfloat16 else "fp16"
    rows = cache[pos].cpu().numpy()
    pn = pos.cpu().numpy()
    rq = ps_oracle.rope(tensor_to_f32(q0).reshape(T, Hq, D), pn, rows, rot, neox, dt)
    rk = ps_oracle.rope(tensor_to_f32(k0).reshape(T, Hkv, D), pn, rows, rot, neox, dt)
    assert np.array_equal(tensor_to_f32(q).reshape(T, Hq, D), rq)
    assert np.array_equal(tensor_to_f32(k).reshape(T, Hkv, D), rk)
    assert torch.equal(v, v0)  # value untouched
    kc_ref, vc_ref = kc0.cpu().float().numpy(), vc0.cpu().float().numpy()
    ps_oracle.kv_append(rk, tensor_to_f32(v0).reshape(T, Hkv, D), kc_ref, vc_ref, slots.cpu().numpy())
    assert np.array_equal(tensor_to_f32(kc), kc_ref) and np.array_equal(tensor_to_f32(vc), vc_ref)


def test_rope_append_flags_positions_outside_the_cache(cuda_device):
    T, Hq, Hkv, D = 4, 4, 2, 128
    q = torch.randn(T, Hq * D, device=cuda_device).to(torch.bfloat16)
    k = torch.randn(T, Hkv * D, device=cuda_device).to(torch.bfloat16)
    v = torch.randn(T, Hkv * D, device=cuda_device).to(torch.bfloat16)
    cache = torch.randn(64, D, device=cuda_device)
    kc = torch.zeros(2, 16, Hkv, D, dtype=torch.bfloat16, device=cuda_device)
    vc = torch.zeros_like(kc)
    pos = torch.tensor([1, 64, 3, -2], dtype=torch.int64, device=cuda_device)
    slots = torch.tensor([0, 1, 2, 3], dtype=torch.int64, device=cuda_device)
    q0 = q.clone()
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    ops.rope_kv_append(q, k, v, pos, cache, True, kc, vc, slots, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) & _lib.PS_DEV_BAD_METADATA
    assert torch.equal(q[1], q0[1]) and torch.equal(q[3], q0[3])  # bad tokens untouched
    assert not torch.equal(q[0], q0[0])
    assert not kc[0, 1].any() and not kc[0, 3].any()  # and not appended


def test_rope_fusion_backend_hook_then_forward(cuda_device):
    """PSRopeAttentionImpl: vLLM's fused RoPE + KV update hook, then forward on
    a decode batch; attention of the rotated query over the updated cache
    matches the oracle (tolerances of the attention tests)."""
    pytest.importorskip("vllm.v1.attention.backend")
    from helpers import assert_attn_close
    from ps_attn import backend as psb
    from ps_attn import workloads

    lens = [40, 300, 17, 1025]
    batch = workloads.make_batch([1] * 4, lens, 16, 8, seed=90)
    g = batch.to(cuda_device)
    T = 4
    maxpos = 2048
    cache = torch.randn(maxpos, 128, device=cuda_device)  # any cos/sin rows
    pos = (g.seq_lens.to(torch.int64) - 1)
    q = g.q.reshape(T, -1).clone()
    k = g.key.reshape(T, -1).clone()
    v = g.value.reshape(T, -1).clone()
    impl = psb.PSRopeAttentionImpl(16, 128, g.softmax_scale, 8, None, None, "auto")
    impl.do_rope_and_kv_cache_update(None, q, k, v, pos, cache, True, g.kv_cache, g.slot_mapping)
    ws = ops.DecodeWorkspace(T, 16, 8, 128, cuda_device)
    md = psb.PSAttentionMetadata(
        num_actual_tokens=T, max_query_len=1, query_start_loc=g.query_start_loc,
        max_seq_len=max(lens), seq_lens=g.seq_lens, block_table=g.block_table,
        slot_mapping=g.slot_mapping, num_decodes=T, num_decode_tokens=T, num_prefills=0,
        workspace=ws)
    out = torch.empty_like(g.q)
    impl.forward(None, q.view(T, 16, 128), k.view(T, 8, 128), v.view(T, 8, 128), g.kv_cache, md, out)
    torch.cuda.synchronize()
    # oracle: rotate on the CPU, append, attend
    rows = cache[pos].cpu().numpy()
    rq = ps_oracle.rope(tensor_to_f32(g.q), pos.cpu().numpy(), rows, 128, True, "bf16")
    rk = ps_oracle.rope(tensor_to_f32(g.key), pos.cpu().numpy(), rows, 128, True, "bf16")
    kc, vc = tensor_to_f32(batch.kv_cache[0]), tensor_to_f32(batch.kv_cache[1])
    ps_oracle.kv_append(rk, tensor_to_f32(g.value), kc, vc, batch.slot_mapping.numpy())
    rout, _ = ps_oracle.paged_attention(rq, kc, vc, batch.block_table.numpy(), batch.seq_lens.numpy(),
                                        batch.query_start_loc.numpy(), batch.softmax_scale)
    assert ws.status() == 0
    assert_attn_close(tensor_to_f32(out), rout)
