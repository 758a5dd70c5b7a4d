"""GPU: decode through the entry point that allocates nothing.

``ps_paged_decode_static_scratch`` serves callers that may not allocate device
memory -- e.g. a backend running inside an inference engine that reserved the
GPU's memory up front and gives none to plugins.  Its scratch is a 16 MiB
array inside the library.  These tests call it through the C ABI several times
in a row and compare the results with the workspace-taking ``ps_paged_decode``
on the same inputs, within the decode tolerances (max-abs 2e-2 / mean-abs 2e-3
on the output, 1e-3 on the LSE).  The array keeps the previous call's
contents: a call that leaves its status word set (an out-of-range block-table
entry, which the kernel records and reads block 0 instead) is followed by a
clean call that must report status 0, which holds only because every call
clears what must start at zero.  The file is collected last.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

from helpers import assert_attn_close, to_np32
from ps_attn import _lib, ops, workloads

pytestmark = pytest.mark.gpu

STATIC_BYTES = 16 << 20


def _static_decode(batch, out, lse, status, key_cache=None, value_cache=None, k_scale=None,
                   v_scale=None, block_table=None):
    lib = _lib.load()
    kc = batch.kv_cache[0] if key_cache is None else key_cache
    vc = batch.kv_cache[1] if value_cache is None else value_cache
    bt = batch.block_table if block_table is None else block_table
    pr = ops._problem(batch.q, kc, vc, bt, batch.seq_lens, batch.query_start_loc, batch.softmax_scale,
                      out, lse, status, k_scale=k_scale, v_scale=v_scale)
    stream = torch.cuda.current_stream(batch.q.device).cuda_stream
    _lib.check(lib.ps_paged_decode_static_scratch(ctypes.byref(pr), stream))


def _decode_batch(cuda_device):
    # config-2 shaped batch plus a long sequence so segments split across warps
    lens = workloads.config_lengths(2)[1][:40] + [9000]
    batch = workloads.make_batch([1] * len(lens), lens, 16, 8, seed=123).to(cuda_device)
    ops.kv_append(batch.key, batch.value, batch.kv_cache[0], batch.kv_cache[1], batch.slot_mapping)
    return batch


def test_static_scratch_decode_matches_workspace_decode(cuda_device):
    batch = _decode_batch(cuda_device)
    B = batch.num_seqs
    ref_out = torch.empty_like(batch.q)
    ref_lse = torch.empty(16, batch.q.shape[0], dtype=torch.float32, device=cuda_device)
    ws = ops.DecodeWorkspace(B, 16, 8, 128, cuda_device)
    ops.paged_decode(batch.q, batch.kv_cache[0], batch.kv_cache[1], batch.block_table,
                     batch.seq_lens, batch.softmax_scale, ref_out, lse=ref_lse,
                     query_start_loc=batch.query_start_loc, workspace=ws)
    status = torch.full((1,), -1, dtype=torch.int32, device=cuda_device)
    for _ in range(2):
        out = torch.full_like(batch.q, float("nan"))
        lse = torch.full_like(ref_lse, float("nan"))
        _static_decode(batch, out, lse, status)
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        assert_attn_close(to_np32(out), to_np32(ref_out), to_np32(lse), to_np32(ref_lse))


def test_each_call_clears_the_previous_calls_status(cuda_device):
    """A call with an out-of-range block-table entry leaves
    PS_DEV_BLOCK_OUT_OF_RANGE in the shared array's status word; the next,
    valid call reports 0 and matches the workspace decode."""
    batch = _decode_batch(cuda_device)
    B = batch.num_seqs
    ref_out = torch.empty_like(batch.q)
    ref_lse = torch.empty(16, B, dtype=torch.float32, device=cuda_device)
    ops.paged_decode(batch.q, batch.kv_cache[0], batch.kv_cache[1], batch.block_table,
                     batch.seq_lens, batch.softmax_scale, ref_out, lse=ref_lse,
                     query_start_loc=batch.query_start_loc,
                     workspace=ops.DecodeWorkspace(B, 16, 8, 128, cuda_device))
    bad_bt = batch.block_table.clone()
    bad_bt[3, 0] = batch.kv_cache.shape[1] + 7  # past the pool: recorded, block 0 read instead
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    out = torch.empty_like(batch.q)
    lse = torch.empty_like(ref_lse)
    for _ in range(2):
        _static_decode(batch, out, lse, status, block_table=bad_bt)
        torch.cuda.synchronize()
        assert int(status.item()) & _lib.PS_DEV_BLOCK_OUT_OF_RANGE
        out2 = torch.full_like(batch.q, float("nan"))
        lse2 = torch.full_like(ref_lse, float("nan"))
        _static_decode(batch, out2, lse2, status)
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        assert_attn_close(to_np32(out2), to_np32(ref_out), to_np32(lse2), to_np32(ref_lse))


def test_static_scratch_fp8_cache(cuda_device):
    """An fp8 (e4m3) cache with per-tensor scales through the static scratch,
    twice, against the workspace decode of the same codes."""
    batch = _decode_batch(cuda_device)
    B = batch.num_seqs
    ks = torch.tensor(0.03, dtype=torch.float32, device=cuda_device)
    vs = torch.tensor(0.02, dtype=torch.float32, device=cuda_device)
    kc = (batch.kv_cache[0].float() / ks).to(torch.float8_e4m3fn).view(torch.uint8)
    vc = (batch.kv_cache[1].float() / vs).to(torch.float8_e4m3fn).view(torch.uint8)
    ref_out = torch.empty_like(batch.q)
    ref_lse = torch.empty(16, B, dtype=torch.float32, device=cuda_device)
    ws = ops.DecodeWorkspace(B, 16, 8, 128, cuda_device)
    ops.paged_decode(batch.q, kc, vc, batch.block_table, batch.seq_lens, batch.softmax_scale, ref_out,
                     lse=ref_lse, query_start_loc=batch.query_start_loc, workspace=ws, k_scale=ks,
                     v_scale=vs)
    status = torch.full((1,), -1, dtype=torch.int32, device=cuda_device)
    for _ in range(2):
        out = torch.full_like(batch.q, float("nan"))
        lse = torch.full_like(ref_lse, float("nan"))
        _static_decode(batch, out, lse, status, key_cache=kc, value_cache=vc, k_scale=ks, v_scale=vs)
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        assert_attn_close(to_np32(out), to_np32(ref_out), to_np32(lse), to_np32(ref_lse))


def test_static_scratch_rejects_oversized_problem(cuda_device):
    lib = _lib.load()
    lens = [16] * 4000  # needs far more than the 16 MiB of library scratch
    batch = workloads.make_batch([1] * len(lens), lens, 8, 8, seed=1, pool_slack=0).to(cuda_device)
    out = torch.empty_like(batch.q)
    pr = ops._problem(batch.q, batch.kv_cache[0], batch.kv_cache[1], batch.block_table,
                      batch.seq_lens, batch.query_start_loc, batch.softmax_scale, out, None)
    rc = lib.ps_paged_decode_static_scratch(ctypes.byref(pr), None)
    assert rc == _lib.PS_ERR_WORKSPACE
    assert b"16 MiB" in lib.ps_last_error()


@pytest.mark.parametrize("fp8", [False, True])
def test_static_scratch_size_limit(cuda_device, fp8):
    """The static scratch takes every problem whose decode scratch fits in
    16 MiB: a split slot per warp of 8 warps per SM with either cache dtype,
    plus one per (sequence, kv head) (352 sequences at 8 KV heads on 148
    SMs)."""
    lib = _lib.load()
    nwarps = torch.cuda.get_device_properties(cuda_device).multi_processor_count * 8
    part_off = 256 + 2 * 4096 * 8 * 4
    limit = (STATIC_BYTES - part_off) // (8 * 129 * 4) - nwarps
    max_seqs = limit // 8
    for n, ok in ((max_seqs, True), (max_seqs + 1, False)):
        batch = workloads.make_batch([1] * n, [40] * n, 16, 8, seed=2, pool_slack=0).to(cuda_device)
        kc, vc = batch.kv_cache[0], batch.kv_cache[1]
        kw = {}
        if fp8:
            kc = torch.zeros(kc.shape, dtype=torch.uint8, device=cuda_device)
            vc = torch.zeros_like(kc)
            one = torch.ones(1, dtype=torch.float32, device=cuda_device)
            kw = dict(k_scale=one, v_scale=one)
        out = torch.empty_like(batch.q)
        pr = ops._problem(batch.q, kc, vc, batch.block_table, batch.seq_lens, batch.query_start_loc,
                          batch.softmax_scale, out, None, **kw)
        rc = lib.ps_paged_decode_static_scratch(ctypes.byref(pr), None)
        torch.cuda.synchronize()
        assert rc == (_lib.PS_OK if ok else _lib.PS_ERR_WORKSPACE), (n, rc)
