"""CPU: the C-ABI library loads, exports every declared symbol and validates
arguments on the host (no kernel is launched here)."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from ps_attn import _lib

HEADER = Path(__file__).resolve().parent.parent / "include" / "ps_attn.h"


def declared_functions():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(ps_[a-z0-9_]+)\s*\(", text)))


def test_header_and_binding_agree():
    assert declared_functions() == sorted(_lib.EXPORTED_SYMBOLS)


def test_library_loads_and_exports_every_symbol():
    lib = _lib.load()
    for name in declared_functions():
        assert hasattr(lib, name), f"{name} missing from libps_attn.so"
    assert lib.ps_abi_version() == _lib.ABI_VERSION


def test_struct_layout_matches_header_order():
    fields = [f for f, _ in _lib.PagedProblem._fields_]
    text = HEADER.read_text()
    body = text[text.index("typedef struct {"):text.index("} ps_paged_problem;")]
    body = re.sub(r"/\*.*?\*/", "", body, flags=re.S)
    names = []
    for decl in body.split(";"):
        decl = decl.strip()
        if not decl or decl.startswith("typedef"):
            decl = decl.replace("typedef struct {", "").strip()
        if not decl:
            continue
        toks = decl.replace("*", " ").replace(",", " ").split()
        # drop the type tokens: everything up to the first field name
        for i, tok in enumerate(toks):
            if tok not in ("const", "void", "int64_t", "int32_t", "float"):
                names.extend(toks[i:])
                break
    assert names == fields


def test_host_validation_errors_without_gpu():
    lib = _lib.load()
    # NULL problem -> invalid argument, message set
    rc = lib.ps_paged_decode(None, None, 0, None)
    assert rc == _lib.PS_ERR_INVALID_ARGUMENT
    assert b"NULL" in lib.ps_last_error()
    # zero tokens is a no-op success, negative is rejected
    args = [None, 0, 0, None, 0, 0, None, None, 0, 0, 0, 1, None, 0, 8, 128, 16, 2, None, None]
    assert lib.ps_kv_append(*args) == _lib.PS_OK
    args[13] = -1
    assert lib.ps_kv_append(*args) == _lib.PS_ERR_INVALID_ARGUMENT
    # unsupported dtype is reported as such (checked before any device query)
    pr = _lib.PagedProblem()
    for f in ("q", "key_cache", "value_cache", "block_table", "seq_lens", "out"):
        setattr(pr, f, 4096)
    pr.num_seqs, pr.dtype, pr.head_size, pr.block_size = 1, _lib.PS_DTYPE_FP32, 128, 16
    pr.num_q_heads, pr.num_kv_heads, pr.num_blocks = 8, 2, 4
    assert lib.ps_paged_decode(ctypes.byref(pr), None, 0, None) == _lib.PS_ERR_UNSUPPORTED
    pr.dtype, pr.head_size = _lib.PS_DTYPE_BF16, 96
    assert lib.ps_paged_decode(ctypes.byref(pr), None, 0, None) == _lib.PS_ERR_UNSUPPORTED
    pr.head_size, pr.block_size = 128, 24
    assert lib.ps_paged_decode(ctypes.byref(pr), None, 0, None) == _lib.PS_ERR_INVALID_ARGUMENT
    pr.block_size, pr.num_q_heads = 16, 7
    assert lib.ps_paged_decode(ctypes.byref(pr), None, 0, None) == _lib.PS_ERR_INVALID_ARGUMENT
    # prefill requires query_start_loc
    pr.num_q_heads = 8
    assert lib.ps_chunked_prefill(ctypes.byref(pr), None) == _lib.PS_ERR_INVALID_ARGUMENT


def test_ops_refuse_cpu_tensors():
    import torch

    from ps_attn import ops

    k = torch.zeros(2, 1, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        ops.kv_append(k, k, torch.zeros(1, 16, 1, 128, dtype=torch.bfloat16),
                      torch.zeros(1, 16, 1, 128, dtype=torch.bfloat16),
                      torch.zeros(2, dtype=torch.int64))


def test_cascade_entry_points_validate_on_the_host():
    lib = _lib.load()
    assert lib.ps_cascade_plan_bytes(-1) == -1
    assert lib.ps_cascade_plan_bytes(4096) == -1  # over the per-launch limit
    # header (32 words) + seq_group + shared_pages (B each) + 3 group arrays (B/2)
    assert lib.ps_cascade_plan_bytes(8) == (32 + 2 * 8 + 3 * 4) * 4
    assert lib.ps_cascade_plan_bytes(1) == (32 + 2 + 3) * 4
    assert lib.ps_cascade_plan_build(None, 8, None, 0, None) == _lib.PS_ERR_INVALID_ARGUMENT
    rc = lib.ps_paged_decode_cascade(None, None, 0, None, 0, None)
    assert rc == _lib.PS_ERR_INVALID_ARGUMENT
    pr = _lib.PagedProblem()
    pr.num_seqs = 3000
    rc = lib.ps_cascade_plan_build(ctypes.byref(pr), 8, ctypes.c_void_p(16), 1 << 20, None)
    assert rc == _lib.PS_ERR_UNSUPPORTED and b"2048" in lib.ps_last_error()
    pr.num_seqs = 4
    rc = lib.ps_cascade_plan_build(ctypes.byref(pr), 0, ctypes.c_void_p(16), 1 << 20, None)
    assert rc == _lib.PS_ERR_INVALID_ARGUMENT
    rc = lib.ps_cascade_plan_build(ctypes.byref(pr), 8, ctypes.c_void_p(16), 8, None)
    assert rc == _lib.PS_ERR_INVALID_ARGUMENT  # buffer too small


def _struct_fields(name):
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    end = text.index("} " + name + ";")
    start = text.rindex("typedef struct {", 0, end) + len("typedef struct {")
    names = []
    for decl in text[start:end].split(";"):
        toks = re.sub(r"\[[^\]]*\]", "", decl).replace("*", " ").replace(",", " ").split()
        for i, tok in enumerate(toks):
            if tok not in ("const", "void", "int64_t", "int32_t", "float"):
                names.extend(toks[i:])
                break
    return names


def test_rope_struct_layout_and_validation():
    assert _struct_fields("ps_rope_append_problem") == [f for f, _ in _lib.RopeAppendProblem._fields_]
    assert _struct_fields("ps_paged_problem") == [f for f, _ in _lib.PagedProblem._fields_]
    lib = _lib.load()
    assert lib.ps_rope_kv_append(None, None) == _lib.PS_ERR_INVALID_ARGUMENT
    pr = _lib.RopeAppendProblem()
    pr.num_tokens = 0
    assert lib.ps_rope_kv_append(ctypes.byref(pr), None) == _lib.PS_OK  # nothing to do
    pr.num_tokens = 4
    assert lib.ps_rope_kv_append(ctypes.byref(pr), None) == _lib.PS_ERR_INVALID_ARGUMENT
    for name in ("query", "key", "value", "key_cache", "value_cache", "slot_mapping", "positions",
                 "cos_sin_cache"):
        setattr(pr, name, 16)
    pr.dtype, pr.cos_sin_dtype = _lib.PS_DTYPE_FP32, _lib.PS_DTYPE_FP32
    assert lib.ps_rope_kv_append(ctypes.byref(pr), None) == _lib.PS_ERR_UNSUPPORTED
    pr.dtype, pr.head_size, pr.rotary_dim = _lib.PS_DTYPE_BF16, 128, 63
    assert lib.ps_rope_kv_append(ctypes.byref(pr), None) == _lib.PS_ERR_INVALID_ARGUMENT
    assert b"rotary_dim" in lib.ps_last_error()


def test_head_gather_struct_and_validation():
    assert _struct_fields("ps_head_gather_problem") == [
        "world", "rank", "num_tokens", "hq_local", "max_tokens", "dtype", "slabs", "out",
        "out_stride_token", "out_stride_head", "status"]
    assert [f for f, _ in _lib.HeadGatherProblem._fields_] == _struct_fields("ps_head_gather_problem")
    lib = _lib.load()
    assert lib.ps_head_gather_slab_bytes(64, 8) == 256 + 64 * 8 * 256
    assert lib.ps_head_gather_slab_bytes(0, 8) == -1
    assert lib.ps_head_gather(None, None) == _lib.PS_ERR_INVALID_ARGUMENT
    hp = _lib.HeadGatherProblem()
    hp.world, hp.rank, hp.num_tokens, hp.hq_local, hp.max_tokens = 9, 0, 4, 8, 8
    hp.dtype = _lib.PS_DTYPE_BF16
    assert lib.ps_head_gather(ctypes.byref(hp), None) == _lib.PS_ERR_INVALID_ARGUMENT
    hp.world = 2
    hp.slabs[0], hp.slabs[1] = 256, 512
    hp.out, hp.out_stride_token, hp.out_stride_head = 1024, 16 * 128, 128
    assert lib.ps_head_gather(ctypes.byref(hp), None) == _lib.PS_ERR_INVALID_ARGUMENT
    assert b"status" in lib.ps_last_error()
    hp.status = 4096
    hp.dtype = _lib.PS_DTYPE_FP32
    assert lib.ps_head_gather(ctypes.byref(hp), None) == _lib.PS_ERR_UNSUPPORTED
    hp.dtype, hp.num_tokens = _lib.PS_DTYPE_BF16, 9  # more rows than the slabs hold
    assert lib.ps_head_gather(ctypes.byref(hp), None) == _lib.PS_ERR_INVALID_ARGUMENT
    assert lib.ps_head_gather_phase(ctypes.byref(hp), 3, None) == _lib.PS_ERR_INVALID_ARGUMENT


def test_fused_decode_head_gather_validation():
    """ps_paged_decode_head_gather: slab size and host-side refusals (no
    kernel launched)."""
    lib = _lib.load()
    # the group's rows [max_tokens, num_q_heads, 128] after the 256-byte header
    assert lib.ps_decode_head_gather_slab_bytes(512, 64) == 256 + 512 * 64 * 256
    assert lib.ps_decode_head_gather_slab_bytes(0, 64) == -1
    assert lib.ps_paged_decode_head_gather(None, None, 0, None, None) == _lib.PS_ERR_INVALID_ARGUMENT
    hp = _lib.HeadGatherProblem()
    hp.world, hp.rank, hp.num_tokens, hp.hq_local, hp.max_tokens = 2, 1, 4, 8, 8
    hp.dtype = _lib.PS_DTYPE_BF16
    hp.slabs[0], hp.slabs[1] = 256, 512
    hp.out, hp.out_stride_token, hp.out_stride_head = 1024, 16 * 128, 128
    hp.status = 4096
    pr = _lib.PagedProblem()
    assert lib.ps_paged_decode_head_gather(None, None, 0, ctypes.byref(hp), None) == _lib.PS_ERR_INVALID_ARGUMENT
    pr.num_q_heads, pr.num_kv_heads, pr.dtype, pr.num_seqs = 16, 2, _lib.PS_DTYPE_BF16, 4
    rc = lib.ps_paged_decode_head_gather(ctypes.byref(pr), None, 0, ctypes.byref(hp), None)
    assert rc == _lib.PS_ERR_INVALID_ARGUMENT and b"hq_local" in lib.ps_last_error()
    pr.num_q_heads = 8
    pr.dtype = _lib.PS_DTYPE_FP16
    rc = lib.ps_paged_decode_head_gather(ctypes.byref(pr), None, 0, ctypes.byref(hp), None)
    assert rc == _lib.PS_ERR_INVALID_ARGUMENT and b"dtype" in lib.ps_last_error()
    pr.dtype, pr.num_seqs = _lib.PS_DTYPE_BF16, 5  # more sequences than the gather's rows
    rc = lib.ps_paged_decode_head_gather(ctypes.byref(pr), None, 0, ctypes.byref(hp), None)
    assert rc == _lib.PS_ERR_INVALID_ARGUMENT
    pr.num_seqs = 0  # every rank must skip an empty step rather than launch
    rc = lib.ps_paged_decode_head_gather(ctypes.byref(pr), None, 0, ctypes.byref(hp), None)
    assert rc == _lib.PS_ERR_INVALID_ARGUMENT and b"empty" in lib.ps_last_error()
