"""GPU: decode through the entry point that allocates nothing.

``ps_paged_decode_static_scratch`` serves callers that may not allocate device
memory -- e.g. a backend running inside an inference engine that reserved the
GPU's memory up front and gives none to plugins.  Its scratch is a 16 MiB
array inside the library.  This test calls it through the C ABI twice in a
row (the array keeps the previous call's contents, so the second call checks
that the entry point clears what must start at zero) and compares both results
with the workspace-taking ``ps_paged_decode`` on the same inputs, within the
decode tolerances (max-abs 2e-2 / mean-abs 2e-3 on the output, 1e-3 on the
LSE).  It lives in its own file, collected last.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

from helpers import assert_attn_close, to_np32
from ps_attn import _lib, ops, workloads

pytestmark = pytest.mark.gpu


def _static_decode(batch, out, lse, status):
    lib = _lib.load()
    pr = ops._problem(batch.q, batch.kv_cache[0], batch.kv_cache[1], batch.block_table,
                      batch.seq_lens, batch.query_start_loc, batch.softmax_scale, out, lse, status)
    stream = torch.cuda.current_stream(batch.q.device).cuda_stream
    _lib.check(lib.ps_paged_decode_static_scratch(ctypes.byref(pr), stream))


def test_static_scratch_decode_matches_workspace_decode(cuda_device):
    # config-2 shaped batch plus a long sequence so segments split across warps
    lens = workloads.config_lengths(2)[1][:40] + [9000]
    batch = workloads.make_batch([1] * len(lens), lens, 16, 8, seed=123).to(cuda_device)
    ops.kv_append(batch.key, batch.value, batch.kv_cache[0], batch.kv_cache[1], batch.slot_mapping)
    ref_out = torch.empty_like(batch.q)
    ref_lse = torch.empty(16, batch.q.shape[0], dtype=torch.float32, device=cuda_device)
    ws = ops.DecodeWorkspace(len(lens), 16, 8, 128, cuda_device)
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


def test_static_scratch_size_limit(cuda_device):
    """The static scratch takes every problem whose decode workspace fits in
    16 MiB: 352 sequences at 8 KV heads on 148 SMs."""
    lib = _lib.load()
    nwarps = torch.cuda.get_device_properties(cuda_device).multi_processor_count * 8
    part_off = 256 + 2 * 4096 * 8 * 4
    limit = ((16 << 20) - part_off) // (8 * 129 * 4) - nwarps
    max_seqs = limit // 8
    for n, ok in ((max_seqs, True), (max_seqs + 1, False)):
        batch = workloads.make_batch([1] * n, [40] * n, 16, 8, seed=2, pool_slack=0).to(cuda_device)
        out = torch.empty_like(batch.q)
        pr = ops._problem(batch.q, batch.kv_cache[0], batch.kv_cache[1], batch.block_table,
                          batch.seq_lens, batch.query_start_loc, batch.softmax_scale, out, None)
        rc = lib.ps_paged_decode_static_scratch(ctypes.byref(pr), None)
        torch.cuda.synchronize()
        assert rc == (_lib.PS_OK if ok else _lib.PS_ERR_WORKSPACE), (n, rc)
