"""CPU: the oracle's e4m3 conversion pinned to torch's float8_e4m3fn (every
value below the overflow boundary, from every bf16 bit pattern at several
scales), its saturation rule, and the fp8 entry points' host validation."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from oracle import ps_oracle
from ps_attn import _lib


@pytest.mark.parametrize("scale", [1.0, 0.37, 3.1, 1.0 / 448.0, 2.0 ** -10])
def test_e4m3_encode_matches_torch_below_overflow(scale):
    x = (np.arange(65536, dtype=np.uint32) << 16).view(np.float32)
    with np.errstate(all="ignore"):
        y = (x / np.float32(scale)).astype(np.float32)
    keep = np.isfinite(y) & (np.abs(y) < 464.0)  # torch turns larger values into NaN
    ref = torch.from_numpy(y[keep]).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(ps_oracle.e4m3_encode(y[keep]), ref)


def test_e4m3_decode_matches_torch_and_saturation():
    codes = np.arange(256, dtype=np.uint8)
    mine = ps_oracle.e4m3_decode(codes)
    ref = torch.from_numpy(codes).view(torch.float8_e4m3fn).float().numpy()
    assert np.array_equal(np.isnan(mine), np.isnan(ref))
    assert np.array_equal(mine[~np.isnan(mine)], ref[~np.isnan(ref)])
    # satfinite: every finite magnitude past 448 stores 448; NaN stays NaN
    big = np.array([448.0, 463.9, 464.0, 1e4, 3e38, -500.0, np.nan], np.float32)
    got = ps_oracle.e4m3_decode(ps_oracle.e4m3_encode(big))
    assert np.array_equal(got[:6], [448, 448, 448, 448, 448, -448]) and np.isnan(got[6])


def test_fp8_append_oracle_round_trip():
    g = np.random.default_rng(0)
    key = g.standard_normal((5, 2, 128)).astype(np.float32)
    val = g.standard_normal((5, 2, 128)).astype(np.float32)
    kc = np.zeros((4, 16, 2, 128), np.uint8)
    vc = np.zeros_like(kc)
    slots = np.array([0, 17, -1, 63, 5])
    ps_oracle.kv_append_fp8(key, val, kc, vc, slots, 0.05, 0.1)
    back = ps_oracle.dequantize_cache(kc, 0.05).reshape(-1, 2, 128)[slots[slots >= 0]]
    # e4m3 keeps 3 mantissa bits: relative error <= 2^-4 for normal values
    ok = np.abs(key[slots >= 0]) > 0.05 * 2.0 ** -6
    rel = np.abs(back - key[slots >= 0]) / np.abs(key[slots >= 0])
    assert (rel[ok] <= 2.0 ** -4 + 1e-7).all()


def test_fp8_entry_points_validate_on_the_host():
    lib = _lib.load()
    args = [None, 0, 0, None, 0, 0, None, None, 0, 0, 0, 1, None, 4, 8, 128, 16,
            _lib.PS_DTYPE_BF16, None, None, None, None]
    assert lib.ps_kv_append_fp8(*args) == _lib.PS_ERR_INVALID_ARGUMENT  # NULL pointers
    args[13] = 0
    assert lib.ps_kv_append_fp8(*args) == _lib.PS_OK  # nothing to do
    args[13] = 4
    for i in (0, 3, 6, 7, 12):
        args[i] = 256
    args[1] = args[4] = 8 * 128
    args[2] = args[5] = 128
    args[8], args[9], args[10] = 16 * 8 * 128, 8 * 128, 128
    args[17] = _lib.PS_DTYPE_FP32
    assert lib.ps_kv_append_fp8(*args) == _lib.PS_ERR_UNSUPPORTED
    args[17] = _lib.PS_DTYPE_BF16
    args[15] = 100  # head_size not a multiple of 8
    assert lib.ps_kv_append_fp8(*args) == _lib.PS_ERR_INVALID_ARGUMENT
    args[15] = 128
    args[10] = 132  # cache rows not 8-byte aligned
    assert lib.ps_kv_append_fp8(*args) == _lib.PS_ERR_INVALID_ARGUMENT
    # an unknown kv_cache_dtype and fp8 caches where no fp8 path is built
    pr = _lib.PagedProblem()
    for name in ("q", "key_cache", "value_cache", "block_table", "seq_lens", "out", "query_start_loc"):
        setattr(pr, name, 256)
    pr.q_stride_token, pr.q_stride_head = 16 * 128, 128
    pr.out_stride_token, pr.out_stride_head = 16 * 128, 128
    pr.cache_stride_block, pr.cache_stride_slot, pr.cache_stride_head = 16 * 8 * 128, 8 * 128, 128
    pr.num_blocks, pr.block_table_stride, pr.max_blocks_per_seq = 8, 4, 4
    pr.num_seqs, pr.num_tokens = 1, 4
    pr.num_q_heads, pr.num_kv_heads, pr.head_size, pr.block_size = 16, 8, 128, 16
    pr.dtype, pr.softmax_scale = _lib.PS_DTYPE_BF16, 0.088
    pr.kv_cache_dtype = 7
    assert lib.ps_chunked_prefill_ws(ctypes.byref(pr), None, 0, None) == _lib.PS_ERR_INVALID_ARGUMENT
    pr.kv_cache_dtype = _lib.PS_KV_FP8_E4M3
    assert lib.ps_chunked_prefill_ws(ctypes.byref(pr), None, 0, None) == _lib.PS_ERR_UNSUPPORTED
    assert b"fp8" in lib.ps_last_error()
