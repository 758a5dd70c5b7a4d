"""GPU: KV append is a bit-exact scatter (vs the oracle, the reference's Triton
goldens and, where vLLM's compiled op loads, vLLM's own reshape_and_cache_flash)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import GOLDEN, build_case, oracle_append
from ps_attn import _lib, ops

pytestmark = pytest.mark.gpu


def _bits(t):
    return t.detach().cpu().contiguous().view(torch.uint8)


@pytest.mark.parametrize("name", ["bf16", "fp32"])
def test_append_matches_triton_golden(cuda_device, name):
    d = np.load(GOLDEN / f"append_{name}.npz")
    dt = torch.bfloat16 if name == "bf16" else torch.float32
    conv = (lambda a: torch.from_numpy(a).view(torch.bfloat16)) if name == "bf16" else torch.from_numpy
    qkv = conv(d["qkv"]).to(cuda_device)
    H, D = d["key_cache_in"].shape[2:]
    key = qkv[:, 4 * D:(4 + H) * D].view(qkv.shape[0], H, D)   # strided token rows
    value = qkv[:, (4 + H) * D:].view(qkv.shape[0], H, D)
    kc = conv(d["key_cache_in"].copy()).to(cuda_device)
    vc = conv(d["value_cache_in"].copy()).to(cuda_device)
    slots = torch.from_numpy(d["slot_mapping"]).to(cuda_device)
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    ops.kv_append(key, value, kc, vc, slots, status=status)
    torch.cuda.synchronize()
    assert kc.dtype == dt
    assert torch.equal(_bits(kc), _bits(conv(d["key_cache_out"])))
    assert torch.equal(_bits(vc), _bits(conv(d["value_cache_out"])))
    assert int(status.item()) == 0


@pytest.mark.parametrize("spec", [
    dict(cfg=2),
    dict(q_lens=[5, 37, 1, 16], seq_lens=[5, 90, 33, 200], num_q_heads=8, num_kv_heads=2, seed=5),
    dict(q_lens=[3, 1], seq_lens=[40, 7], num_q_heads=4, num_kv_heads=1, block_size=32, seed=6),
])
def test_append_matches_oracle(cuda_device, spec):
    batch = build_case(spec)
    kc_ref, vc_ref = oracle_append(batch)
    g = batch.to(cuda_device)
    ops.kv_append(g.key, g.value, g.kv_cache[0], g.kv_cache[1], g.slot_mapping)
    torch.cuda.synchronize()
    assert torch.equal(_bits(g.kv_cache[0]), _bits(kc_ref))
    assert torch.equal(_bits(g.kv_cache[1]), _bits(vc_ref))


def test_append_skips_negative_and_flags_out_of_range(cuda_device):
    nb, bs, h, d = 4, 16, 2, 128
    kc = torch.zeros(nb, bs, h, d, dtype=torch.bfloat16, device=cuda_device)
    vc = torch.zeros_like(kc)
    key = torch.randn(4, h, d, dtype=torch.bfloat16, device=cuda_device)
    val = torch.randn_like(key)
    slots = torch.tensor([-1, 5, nb * bs + 3, -7], dtype=torch.int64, device=cuda_device)
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    ops.kv_append(key, val, kc, vc, slots, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) & _lib.PS_DEV_SLOT_OUT_OF_RANGE
    assert torch.equal(kc.view(-1, h, d)[5], key[1])
    assert torch.equal(vc.view(-1, h, d)[5], val[1])
    kc.view(-1, h, d)[5] = 0
    vc.view(-1, h, d)[5] = 0
    assert not kc.any() and not vc.any()


def test_append_handles_unaligned_rows_with_narrow_vectors(cuda_device):
    # head_size 68 bf16 -> 136-byte rows: 16-byte vectors do not divide, 8-byte ones do
    nb, bs, h, d = 3, 16, 3, 68
    kc = torch.zeros(nb, bs, h, d, dtype=torch.bfloat16, device=cuda_device)
    vc = torch.zeros_like(kc)
    key = torch.randn(5, h, d, dtype=torch.bfloat16, device=cuda_device)
    val = torch.randn_like(key)
    slots = torch.tensor([0, 17, 47, -1, 30], dtype=torch.int64, device=cuda_device)
    ops.kv_append(key, val, kc, vc, slots)
    torch.cuda.synchronize()
    ref_k = torch.zeros_like(kc)
    ref_v = torch.zeros_like(vc)
    ok = slots >= 0
    ref_k.view(-1, h, d)[slots[ok]] = key[ok]
    ref_v.view(-1, h, d)[slots[ok]] = val[ok]
    assert torch.equal(kc, ref_k) and torch.equal(vc, ref_v)


def test_append_matches_vllm_compiled_op(cuda_device):
    try:
        from vllm import _custom_ops as vops  # noqa: F401
        fn = torch.ops._C_cache_ops.reshape_and_cache_flash
    except Exception as e:  # pragma: no cover - depends on the box's vLLM build
        pytest.skip(f"vLLM compiled cache ops unavailable: {e}")
    batch = build_case(dict(cfg=2)).to(cuda_device)
    kc1, vc1 = batch.kv_cache[0].clone(), batch.kv_cache[1].clone()
    kc2, vc2 = batch.kv_cache[0].clone(), batch.kv_cache[1].clone()
    one = torch.ones((), dtype=torch.float32, device=cuda_device)
    fn(batch.key, batch.value, kc1, vc1, batch.slot_mapping, "auto", one, one)
    ops.kv_append(batch.key, batch.value, kc2, vc2, batch.slot_mapping)
    torch.cuda.synchronize()
    assert torch.equal(_bits(kc1), _bits(kc2)) and torch.equal(_bits(vc1), _bits(vc2))
