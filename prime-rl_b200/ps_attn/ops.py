"""Torch-facing ops over libps_attn.so.

These functions mirror the two GPU calls vLLM's FlashAttention backend makes
per decoder layer and keep their argument meaning:

* :func:`kv_append` -- ``reshape_and_cache_flash(key, value, key_cache,
  value_cache, slot_mapping, ...)`` (``vllm/_custom_ops.py:2591-2610``);
* :func:`paged_attention` -- ``flash_attn_varlen_func(q, k_cache, v_cache, out,
  cu_seqlens_q, max_seqlen_q, seqused_k, max_seqlen_k, softmax_scale,
  causal=True, block_table=...)`` as called at
  ``vllm/v1/attention/backends/flash_attn.py:796-817``.  It dispatches to
  :func:`paged_decode` (``max_seqlen_q == 1``) or :func:`chunked_prefill`.

Tensors stay on the device; the work is enqueued on the current CUDA stream;
nothing here synchronises or allocates except :class:`DecodeWorkspace`
construction.  All validation failures raise :class:`ps_attn._lib.PSError` or
``ValueError``; there is no non-CUDA path.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib

_DTYPES = {
    torch.float16: _lib.PS_DTYPE_FP16,
    torch.bfloat16: _lib.PS_DTYPE_BF16,
    torch.float32: _lib.PS_DTYPE_FP32,
}


def _stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(*tensors):
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise ValueError("ps_attn ops take CUDA tensors only (no CPU path)")


FP8_CACHE_DTYPES = (torch.uint8, torch.float8_e4m3fn)


def is_fp8_cache(cache: torch.Tensor) -> bool:
    """An fp8 (e4m3) KV cache: uint8 codes or torch.float8_e4m3fn."""
    return cache.dtype in FP8_CACHE_DTYPES


def _scale_ptr(scale):
    if scale is None:
        return None
    if scale.dtype != torch.float32 or not scale.is_cuda or scale.numel() != 1:
        raise ValueError("k_scale / v_scale must be one-element CUDA float32 tensors")
    return scale.data_ptr()


def kv_append(key: torch.Tensor, value: torch.Tensor, key_cache: torch.Tensor,
              value_cache: torch.Tensor, slot_mapping: torch.Tensor,
              status: torch.Tensor | None = None, k_scale: torch.Tensor | None = None,
              v_scale: torch.Tensor | None = None) -> None:
    """Write ``key``/``value`` rows into the paged cache at ``slot_mapping``.

    key, value: [T', Hkv, D] (T' >= len(slot_mapping)); key_cache,
    value_cache: [num_blocks, block_size, Hkv, D]; slot_mapping: int64 [T].
    Negative slots are skipped.  Bit-exact copy; for an fp8 cache (uint8 or
    float8_e4m3fn) the rows are stored as e4m3(x / k_scale) and
    e4m3(x / v_scale) (``reshape_and_cache_flash`` with kv_cache_dtype "fp8";
    scales: one-element float32 device tensors, None = 1).
    """
    lib = _lib.load()
    _require_cuda(key, value, key_cache, value_cache, slot_mapping)
    if slot_mapping.dtype != torch.int64:
        raise ValueError("slot_mapping must be int64")
    fp8 = is_fp8_cache(key_cache)
    if fp8:
        if value_cache.dtype != key_cache.dtype or key.dtype != value.dtype or \
                key.dtype not in (torch.float16, torch.bfloat16):
            raise ValueError("fp8 cache: fp16/bf16 key and value rows, both caches fp8")
    elif key.dtype != key_cache.dtype or value.dtype != value_cache.dtype or key.dtype != value.dtype:
        raise ValueError("key/value/cache dtypes must match")
    if key_cache.stride() != value_cache.stride() or key_cache.shape != value_cache.shape:
        raise ValueError("key_cache and value_cache must have the same shape and strides")
    if key.stride(-1) != 1 or value.stride(-1) != 1 or key_cache.stride(-1) != 1:
        raise ValueError("last dimension must be contiguous")
    if not slot_mapping.is_contiguous():
        raise ValueError("slot_mapping must be contiguous")
    T = slot_mapping.shape[0]
    if key.shape[0] < T or value.shape[0] < T:
        raise ValueError("key/value have fewer rows than slot_mapping")
    nb, bs, hkv, d = key_cache.shape
    if key.shape[1:] != (hkv, d) or value.shape[1:] != (hkv, d):
        raise ValueError(f"key/value shape {tuple(key.shape)} does not match cache {tuple(key_cache.shape)}")
    if fp8:
        _lib.check(lib.ps_kv_append_fp8(
            key.data_ptr(), key.stride(0), key.stride(1),
            value.data_ptr(), value.stride(0), value.stride(1),
            key_cache.data_ptr(), value_cache.data_ptr(),
            key_cache.stride(0), key_cache.stride(1), key_cache.stride(2), nb,
            slot_mapping.data_ptr(), T, hkv, d, bs, _DTYPES[key.dtype],
            _scale_ptr(k_scale), _scale_ptr(v_scale),
            status.data_ptr() if status is not None else None,
            _stream_ptr(key.device)))
        return
    _lib.check(lib.ps_kv_append(
        key.data_ptr(), key.stride(0), key.stride(1),
        value.data_ptr(), value.stride(0), value.stride(1),
        key_cache.data_ptr(), value_cache.data_ptr(),
        key_cache.stride(0), key_cache.stride(1), key_cache.stride(2), nb,
        slot_mapping.data_ptr(), T, hkv, d, bs, key.element_size(),
        status.data_ptr() if status is not None else None,
        _stream_ptr(key.device)))


def rope_kv_append(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                   positions: torch.Tensor, cos_sin_cache: torch.Tensor, is_neox: bool,
                   key_cache: torch.Tensor, value_cache: torch.Tensor,
                   slot_mapping: torch.Tensor, status: torch.Tensor | None = None) -> None:
    """Rotary embedding of ``query``/``key`` in place, then the KV append of the
    rotated key and ``value`` (``do_rope_and_kv_cache_update``'s contract).

    query [T, Hq*D] or [T, Hq, D]; key, value [T, Hkv*D] or [T, Hkv, D];
    positions int64 [T]; cos_sin_cache [max_position, rotary_dim] (fp32 or the
    model dtype; cos half then sin half); caches [num_blocks, block_size, Hkv,
    D]; slot_mapping int64 [T] (negative: no cache write).  Bit-identical to
    vLLM's torch-native rotary embedding followed by ``kv_append``.
    """
    lib = _lib.load()
    _require_cuda(query, key, value, positions, cos_sin_cache, key_cache, value_cache, slot_mapping)
    nb, bs, hkv, d = key_cache.shape
    T = slot_mapping.shape[0]
    if positions.dtype != torch.int64 or slot_mapping.dtype != torch.int64:
        raise ValueError("positions and slot_mapping must be int64")
    if positions.numel() < T or not positions.is_contiguous() or not slot_mapping.is_contiguous():
        raise ValueError("positions must hold a position per token; both contiguous")
    q3 = query.view(query.shape[0], -1, d)
    k3 = key.view(key.shape[0], -1, d)
    v3 = value.view(value.shape[0], -1, d)
    if k3.shape[1] != hkv or v3.shape[1] != hkv or q3.shape[0] < T or k3.shape[0] < T:
        raise ValueError("query/key/value shapes do not match the cache")
    dtype = query.dtype
    if dtype not in (torch.bfloat16, torch.float16) or key.dtype != dtype or value.dtype != dtype \
            or key_cache.dtype != dtype or value_cache.dtype != dtype:
        raise ValueError("query, key, value and caches must share one fp16/bf16 dtype")
    if cos_sin_cache.dtype not in (torch.float32, dtype) or cos_sin_cache.stride(-1) != 1:
        raise ValueError("cos_sin_cache must be fp32 or the model dtype, rows contiguous")
    if key_cache.stride() != value_cache.stride() or key_cache.stride(-1) != 1:
        raise ValueError("key_cache and value_cache must share strides, last dim contiguous")
    if q3.stride(-1) != 1 or k3.stride(-1) != 1 or v3.stride(-1) != 1:
        raise ValueError("last dimension must be contiguous")
    pr = _lib.RopeAppendProblem()
    pr.query = q3.data_ptr()
    pr.query_stride_token, pr.query_stride_head = q3.stride(0), q3.stride(1)
    pr.key = k3.data_ptr()
    pr.key_stride_token, pr.key_stride_head = k3.stride(0), k3.stride(1)
    pr.value = v3.data_ptr()
    pr.value_stride_token, pr.value_stride_head = v3.stride(0), v3.stride(1)
    pr.key_cache = key_cache.data_ptr()
    pr.value_cache = value_cache.data_ptr()
    pr.cache_stride_block, pr.cache_stride_slot, pr.cache_stride_head = key_cache.stride()[:3]
    pr.num_blocks = nb
    pr.block_size = bs
    pr.slot_mapping = slot_mapping.data_ptr()
    pr.positions = positions.data_ptr()
    pr.cos_sin_cache = cos_sin_cache.data_ptr()
    pr.cos_sin_stride = cos_sin_cache.stride(0)
    pr.max_position = cos_sin_cache.shape[0]
    pr.cos_sin_dtype = _DTYPES[cos_sin_cache.dtype]
    pr.rotary_dim = cos_sin_cache.shape[-1]
    pr.is_neox = int(bool(is_neox))
    pr.num_tokens = T
    pr.num_q_heads = q3.shape[1]
    pr.num_kv_heads = hkv
    pr.head_size = d
    pr.dtype = _DTYPES[dtype]
    if status is not None:
        pr.status = status.data_ptr()
    _lib.check(lib.ps_rope_kv_append(ctypes.byref(pr), _stream_ptr(query.device)))


class DecodeWorkspace:
    """Fixed-size device workspace for :func:`paged_decode`.

    Sized for ``max_num_seqs`` once (independent of sequence lengths, so one
    buffer serves every step and every CUDA-graph replay) and zeroed at
    creation; the kernel leaves its counters at zero.  ``status()`` reads and
    ``clear_status()`` resets the device status word (PS_DEV_* bits).
    """

    def __init__(self, max_num_seqs: int, num_q_heads: int, num_kv_heads: int,
                 head_size: int, device: torch.device | str | int | None = None,
                 cascade: bool = False):
        lib = _lib.load()
        dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        if dev.type != "cuda":
            raise ValueError("DecodeWorkspace lives on a CUDA device")
        with torch.cuda.device(dev):
            nbytes = lib.ps_paged_decode_workspace_size(max_num_seqs, num_q_heads, num_kv_heads, head_size)
            if cascade:  # serves both kinds of call: the larger size
                nbytes = max(nbytes, lib.ps_paged_decode_cascade_workspace_size(
                    max_num_seqs, num_q_heads, num_kv_heads, head_size))
        if nbytes < 0:
            _lib.check(_lib.PS_ERR_INVALID_ARGUMENT)
        self.cascade = cascade
        self.max_num_seqs = max_num_seqs
        self.num_q_heads = num_q_heads
        self.num_kv_heads = num_kv_heads
        self.nbytes = int(nbytes)
        self.buffer = torch.zeros(self.nbytes, dtype=torch.uint8, device=dev)

    def status(self) -> int:
        return int(self.buffer[:4].view(torch.int32).item())

    def clear_status(self) -> None:
        self.buffer[:4].zero_()


_WS_CACHE: dict = {}


def get_workspace(num_seqs: int, num_q_heads: int, num_kv_heads: int, head_size: int,
                  device: torch.device, cascade: bool = False) -> DecodeWorkspace:
    """Process-wide workspace per (device, heads, kind), grown to the largest batch seen."""
    key = (device.index, num_q_heads, num_kv_heads, head_size, cascade)
    ws = _WS_CACHE.get(key)
    if ws is None or ws.max_num_seqs < num_seqs:
        cap = max(num_seqs, 256 if ws is None else 2 * ws.max_num_seqs)
        if cascade:
            cap = min(cap, CASCADE_MAX_SEQS)
        ws = DecodeWorkspace(cap, num_q_heads, num_kv_heads, head_size, device, cascade=cascade)
        _WS_CACHE[key] = ws
    return ws


CASCADE_MAX_SEQS = 2048
PLAN_HEADER_WORDS = 32


class CascadePlan:
    """Device buffer of a shared-prefix plan (``ps_cascade_plan_build``).

    Sized for up to ``max_num_seqs`` sequences and zeroed once; rebuilt in
    place by :func:`cascade_plan` for each batch (once per step, shared by all
    layers).  ``num_seqs`` is the batch the current contents describe.
    """

    def __init__(self, max_num_seqs: int, device: torch.device | str | int | None = None):
        lib = _lib.load()
        if not 0 <= max_num_seqs <= CASCADE_MAX_SEQS:
            raise ValueError(f"cascade plans hold at most {CASCADE_MAX_SEQS} sequences")
        dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        nbytes = lib.ps_cascade_plan_bytes(max(max_num_seqs, 1))
        if nbytes < 0:
            _lib.check(_lib.PS_ERR_INVALID_ARGUMENT)
        self.max_num_seqs = max_num_seqs
        self.nbytes = int(nbytes)
        self.buffer = torch.zeros(self.nbytes // 4, dtype=torch.int32, device=dev)
        self.num_seqs = 0

    def views(self) -> dict:
        """The plan's arrays for the batch it was last built for (device tensors)."""
        B = self.num_seqs
        gm = max(1, B // 2)
        w = self.buffer
        o = PLAN_HEADER_WORDS
        return {
            "num_groups": w[0:1],
            "seq_group": w[o:o + B],
            "group_first": w[o + B:o + B + gm],
            "group_size": w[o + B + gm:o + B + 2 * gm],
            "group_pages": w[o + B + 2 * gm:o + B + 3 * gm],
            "shared_pages": w[o + B + 3 * gm:o + 2 * B + 3 * gm],
        }


def cascade_plan(block_table: torch.Tensor, seq_lens: torch.Tensor, num_q_heads: int,
                 num_kv_heads: int, block_size: int, query_start_loc: torch.Tensor | None = None,
                 min_shared_pages: int = 8, plan: CascadePlan | None = None) -> CascadePlan:
    """Find groups of adjacent decode sequences with identical leading pages.

    Enqueued on the current stream (no host synchronisation).  The result is
    valid for any later :func:`paged_decode` call on the same block_table,
    seq_lens and query_start_loc; pass it as ``cascade=``.
    """
    lib = _lib.load()
    _require_cuda(block_table, seq_lens, query_start_loc)
    if block_table.dtype != torch.int32 or seq_lens.dtype != torch.int32:
        raise ValueError("block_table and seq_lens must be int32")
    if block_table.stride(-1) != 1 or not seq_lens.is_contiguous():
        raise ValueError("block_table rows and seq_lens must be contiguous")
    B = seq_lens.shape[0]
    if plan is None:
        plan = CascadePlan(B, seq_lens.device)
    elif plan.max_num_seqs < B:
        raise ValueError(f"plan sized for {plan.max_num_seqs} sequences < {B}")
    pr = _lib.PagedProblem()
    pr.block_table = block_table.data_ptr()
    pr.block_table_stride = block_table.stride(0)
    pr.max_blocks_per_seq = block_table.shape[1]
    pr.seq_lens = seq_lens.data_ptr()
    pr.query_start_loc = query_start_loc.data_ptr() if query_start_loc is not None else None
    pr.num_seqs = B
    pr.num_q_heads = num_q_heads
    pr.num_kv_heads = num_kv_heads
    pr.head_size = 128
    pr.block_size = block_size
    _lib.check(lib.ps_cascade_plan_build(ctypes.byref(pr), int(min_shared_pages),
                                         plan.buffer.data_ptr(), plan.nbytes,
                                         _stream_ptr(seq_lens.device)))
    plan.num_seqs = B
    return plan


def _problem(q, key_cache, value_cache, block_table, seq_lens, query_start_loc,
             softmax_scale, out, lse, status=None, k_scale=None, v_scale=None) -> _lib.PagedProblem:
    _require_cuda(q, key_cache, value_cache, block_table, seq_lens, out, query_start_loc, lse)
    if q.dtype not in (torch.float16, torch.bfloat16):
        raise ValueError(f"attention dtype {q.dtype} unsupported (fp16/bf16)")
    fp8 = is_fp8_cache(key_cache)
    if fp8:
        if value_cache.dtype != key_cache.dtype or out.dtype != q.dtype:
            raise ValueError("fp8 cache: both caches fp8, out in the query dtype")
    elif key_cache.dtype != q.dtype or value_cache.dtype != q.dtype or out.dtype != q.dtype:
        raise ValueError("q, caches and out must share one dtype")
    if key_cache.stride() != value_cache.stride() or key_cache.shape != value_cache.shape:
        raise ValueError("key_cache and value_cache must have the same shape and strides")
    if block_table.dtype != torch.int32 or seq_lens.dtype != torch.int32:
        raise ValueError("block_table and seq_lens must be int32")
    if query_start_loc is not None and query_start_loc.dtype != torch.int32:
        raise ValueError("query_start_loc must be int32")
    if block_table.stride(-1) != 1 or not seq_lens.is_contiguous():
        raise ValueError("block_table rows and seq_lens must be contiguous")
    if q.stride(-1) != 1 or out.stride(-1) != 1 or key_cache.stride(-1) != 1:
        raise ValueError("last dimension must be contiguous")
    if lse is not None and lse.dtype != torch.float32:
        raise ValueError("lse must be float32 [num_q_heads, num_tokens]")
    nb, bs, hkv, d = key_cache.shape
    hq = q.shape[1]
    pr = _lib.PagedProblem()
    pr.q = q.data_ptr()
    pr.q_stride_token, pr.q_stride_head = q.stride(0), q.stride(1)
    pr.key_cache = key_cache.data_ptr()
    pr.value_cache = value_cache.data_ptr()
    pr.cache_stride_block, pr.cache_stride_slot, pr.cache_stride_head = key_cache.stride()[:3]
    pr.num_blocks = nb
    pr.block_table = block_table.data_ptr()
    pr.block_table_stride = block_table.stride(0)
    pr.max_blocks_per_seq = block_table.shape[1]
    pr.seq_lens = seq_lens.data_ptr()
    pr.query_start_loc = query_start_loc.data_ptr() if query_start_loc is not None else None
    pr.num_seqs = seq_lens.shape[0]
    pr.out = out.data_ptr()
    pr.out_stride_token, pr.out_stride_head = out.stride(0), out.stride(1)
    if lse is not None:
        pr.lse = lse.data_ptr()
        pr.lse_stride_head, pr.lse_stride_token = lse.stride(0), lse.stride(1)
    pr.num_q_heads = hq
    pr.num_kv_heads = hkv
    pr.head_size = d
    pr.block_size = bs
    pr.dtype = _DTYPES[q.dtype]
    pr.softmax_scale = float(softmax_scale)
    if out.shape[0] < q.shape[0]:
        raise ValueError("out has fewer rows than q")
    pr.num_tokens = q.shape[0]
    if status is not None:
        if status.dtype != torch.int32 or not status.is_cuda:
            raise ValueError("status must be a CUDA int32 tensor")
        pr.status = status.data_ptr()
    if fp8:
        pr.kv_cache_dtype = _lib.PS_KV_FP8_E4M3
    pr.k_scale = _scale_ptr(k_scale)
    pr.v_scale = _scale_ptr(v_scale)
    return pr


def paged_decode(q: torch.Tensor, key_cache: torch.Tensor, value_cache: torch.Tensor,
                 block_table: torch.Tensor, seq_lens: torch.Tensor, softmax_scale: float,
                 out: torch.Tensor, lse: torch.Tensor | None = None,
                 query_start_loc: torch.Tensor | None = None,
                 workspace: DecodeWorkspace | None = None,
                 new_key: torch.Tensor | None = None, new_value: torch.Tensor | None = None,
                 slot_mapping: torch.Tensor | None = None,
                 cascade: CascadePlan | None = None, k_scale: torch.Tensor | None = None,
                 v_scale: torch.Tensor | None = None, out_address: int | None = None,
                 head_gather: "_lib.HeadGatherProblem | None" = None) -> torch.Tensor:
    """Decode attention, one query row per sequence, written into ``out``.

    q/out: [T, Hq, D]; caches [num_blocks, block_size, Hkv, D]; block_table
    int32 [B, P]; seq_lens int32 [B] (including the new token);
    query_start_loc int32 [B+1] or None (row b for sequence b); lse fp32
    [Hq, T] or None (natural log).

    ``new_key``/``new_value`` [T, Hkv, D] + ``slot_mapping`` int64 [T] fuse the
    KV append of the decode tokens into the same launch (same result as
    :func:`kv_append` followed by this call without them).

    ``cascade``: a :class:`CascadePlan` built by :func:`cascade_plan` for this
    batch; shared prefixes are then read once per group pass (same outputs).
    The workspace must then be a cascade workspace.

    fp8 caches (uint8 codes or float8_e4m3fn): attention over code * k_scale
    and code * v_scale (one-element float32 device tensors, None = 1); the
    fused append stores e4m3(x / scale).

    ``out_address``: write the output rows to this device address instead,
    contiguous [T, Hq, D] in ``out``'s dtype (``out`` then only supplies the
    dtype and shape) -- a peer-memory slab for :mod:`ps_attn.sharding`'s
    NVLink head gather.

    ``head_gather``: a filled ``ps_head_gather_problem`` -- this call is then
    one rank's part of a KV-head-sharded group and runs
    ``ps_paged_decode_head_gather`` (the group's rows land in
    ``head_gather.out`` on every rank; ``out`` only supplies shape and dtype).
    Used by :class:`ps_attn.sharding.FusedHeadGather`.
    """
    lib = _lib.load()
    B = seq_lens.shape[0]
    if workspace is None:
        workspace = get_workspace(B, q.shape[1], key_cache.shape[2], key_cache.shape[3], q.device,
                                  cascade=cascade is not None)
    elif workspace.max_num_seqs < B:
        raise ValueError(f"workspace sized for {workspace.max_num_seqs} sequences < {B}")
    if cascade is not None and cascade.num_seqs != B:
        raise ValueError(f"cascade plan built for {cascade.num_seqs} sequences, call has {B}")
    pr = _problem(q, key_cache, value_cache, block_table, seq_lens, query_start_loc,
                  softmax_scale, out, lse, k_scale=k_scale, v_scale=v_scale)
    if out_address is not None:
        if out_address % 16:
            raise ValueError("out_address must be 16-byte aligned")
        pr.out = out_address
        pr.out_stride_token, pr.out_stride_head = q.shape[1] * q.shape[2], q.shape[2]
    if new_key is not None:
        _require_cuda(new_key, new_value, slot_mapping)
        if new_value is None or slot_mapping is None:
            raise ValueError("fused append needs new_key, new_value and slot_mapping")
        if slot_mapping.dtype != torch.int64 or not slot_mapping.is_contiguous():
            raise ValueError("slot_mapping must be contiguous int64")
        if new_key.dtype != q.dtype or new_value.dtype != q.dtype:
            raise ValueError("new key/value must have the query dtype")
        hkv, d = key_cache.shape[2], key_cache.shape[3]
        if new_key.shape[1:] != (hkv, d) or new_value.shape[1:] != (hkv, d):
            raise ValueError("new key/value shape does not match the cache")
        if new_key.stride(-1) != 1 or new_value.stride(-1) != 1:
            raise ValueError("last dimension must be contiguous")
        if slot_mapping.shape[0] < q.shape[0] or new_key.shape[0] < q.shape[0]:
            raise ValueError("fused append needs a key/value row and a slot per query row")
        pr.new_key = new_key.data_ptr()
        pr.new_key_stride_token, pr.new_key_stride_head = new_key.stride(0), new_key.stride(1)
        pr.new_value = new_value.data_ptr()
        pr.new_value_stride_token, pr.new_value_stride_head = new_value.stride(0), new_value.stride(1)
        pr.slot_mapping = slot_mapping.data_ptr()
    if head_gather is not None:
        if cascade is not None or out_address is not None:
            raise ValueError("the fused head gather runs the plain decode into its own output")
        _lib.check(lib.ps_paged_decode_head_gather(ctypes.byref(pr), workspace.buffer.data_ptr(),
                                                   workspace.nbytes, ctypes.byref(head_gather),
                                                   _stream_ptr(q.device)))
    elif cascade is not None:
        _lib.check(lib.ps_paged_decode_cascade(ctypes.byref(pr), cascade.buffer.data_ptr(),
                                               cascade.nbytes, workspace.buffer.data_ptr(),
                                               workspace.nbytes, _stream_ptr(q.device)))
    else:
        _lib.check(lib.ps_paged_decode(ctypes.byref(pr), workspace.buffer.data_ptr(),
                                       workspace.nbytes, _stream_ptr(q.device)))
    return out


def dequant_gather(key_cache: torch.Tensor, value_cache: torch.Tensor, block_table: torch.Tensor,
                   seq_lens: torch.Tensor, max_pages: int, dtype: torch.dtype,
                   k_scale: torch.Tensor | None = None, v_scale: torch.Tensor | None = None,
                   status: torch.Tensor | None = None):
    """The pages ``seq_lens`` covers of an fp8 cache, dequantized into a
    16-bit scratch cache: returns (key, value [B * max_pages, bs, Hkv, D] of
    ``dtype``, block table [B, max_pages] int32 into them).  Pages past a
    sequence's length are left uninitialised (never read).  Without scales
    the scratch holds the e4m3 values exactly (attend over it with the
    scales); with them, code * scale rounded to ``dtype``."""
    lib = _lib.load()
    _require_cuda(key_cache, value_cache, block_table, seq_lens)
    if not is_fp8_cache(key_cache) or value_cache.dtype != key_cache.dtype:
        raise ValueError("dequant_gather reads an fp8 cache")
    B = seq_lens.shape[0]
    nb, bs, hkv, d = key_cache.shape
    dev = key_cache.device
    kd = torch.empty(B * max_pages, bs, hkv, d, dtype=dtype, device=dev)
    vd = torch.empty_like(kd)
    bt = torch.arange(B * max_pages, dtype=torch.int32, device=dev).view(B, max_pages)
    if B == 0 or max_pages == 0:
        return kd, vd, bt
    q_like = torch.empty(1, 1, d, dtype=dtype, device=dev)
    pr = _problem(q_like, key_cache, value_cache, block_table, seq_lens, None, 1.0, q_like, None,
                  status=status, k_scale=k_scale, v_scale=v_scale)
    _lib.check(lib.ps_kv_dequant_gather(ctypes.byref(pr), max_pages, kd.data_ptr(), vd.data_ptr(),
                                        _stream_ptr(dev)))
    return kd, vd, bt


def merge_attn_states(output: torch.Tensor, prefix_output: torch.Tensor, prefix_lse: torch.Tensor,
                      suffix_output: torch.Tensor, suffix_lse: torch.Tensor,
                      output_lse: torch.Tensor | None = None) -> torch.Tensor:
    """vLLM's ``merge_attn_states`` (``vllm/v1/attention/ops/merge_attn_states.py:9``):
    two partial attentions of the same rows over disjoint keys, outputs
    [T, H, D] and LSEs [H, T] (fp32, contiguous), into ``output`` (may alias
    an input) and ``output_lse``."""
    lib = _lib.load()
    _require_cuda(output, prefix_output, prefix_lse, suffix_output, suffix_lse, output_lse)
    T, H, D = output.shape
    for t in (prefix_output, suffix_output):
        if t.dtype != output.dtype or tuple(t.shape) != (T, H, D) or t.stride(-1) != 1:
            raise ValueError("prefix/suffix outputs must match output [T, H, D]")
    for t in (prefix_lse, suffix_lse) + ((output_lse,) if output_lse is not None else ()):
        if t.dtype != torch.float32 or tuple(t.shape) != (H, T) or not t.is_contiguous():
            raise ValueError("LSEs must be contiguous float32 [H, T]")
    _lib.check(lib.ps_merge_attn_states(
        prefix_output.data_ptr(), prefix_output.stride(0), prefix_output.stride(1), prefix_lse.data_ptr(),
        suffix_output.data_ptr(), suffix_output.stride(0), suffix_output.stride(1), suffix_lse.data_ptr(),
        output.data_ptr(), output.stride(0), output.stride(1),
        output_lse.data_ptr() if output_lse is not None else None,
        T, H, D, _DTYPES[output.dtype], _stream_ptr(output.device)))
    return output


def chunked_prefill(q: torch.Tensor, key_cache: torch.Tensor, value_cache: torch.Tensor,
                    block_table: torch.Tensor, seq_lens: torch.Tensor,
                    query_start_loc: torch.Tensor, softmax_scale: float, out: torch.Tensor,
                    lse: torch.Tensor | None = None,
                    status: torch.Tensor | None = None,
                    workspace: "DecodeWorkspace | None" = None,
                    k_scale: torch.Tensor | None = None,
                    v_scale: torch.Tensor | None = None) -> torch.Tensor:
    """Causal (bottom-right) varlen attention over the paged cache; any q_len >= 1.

    ``k_scale``/``v_scale`` (one-element float32 device tensors): the cache
    is read as K * k_scale, V * v_scale -- attention over the unscaled
    scratch of :func:`dequant_gather` with an fp8 cache's scales.

    ``query_start_loc`` [B+1] holds absolute row offsets into ``q``/``out``
    (a slice of a larger batch's offsets is fine).  ``status`` (int32 [1],
    optional) receives PS_DEV_* bits from device-side checks.  With a
    ``workspace`` (a :class:`DecodeWorkspace` serves) the work units are
    handed out dynamically (``ps_chunked_prefill_ws``).
    """
    lib = _lib.load()
    if query_start_loc is None:
        raise ValueError("chunked_prefill needs query_start_loc")
    pr = _problem(q, key_cache, value_cache, block_table, seq_lens, query_start_loc,
                  softmax_scale, out, lse, status, k_scale=k_scale, v_scale=v_scale)
    if workspace is not None:
        _lib.check(lib.ps_chunked_prefill_ws(ctypes.byref(pr), workspace.buffer.data_ptr(),
                                             workspace.nbytes, _stream_ptr(q.device)))
    else:
        _lib.check(lib.ps_chunked_prefill(ctypes.byref(pr), _stream_ptr(q.device)))
    return out


def paged_attention(q, key_cache, value_cache, out, query_start_loc, max_query_len, seq_lens,
                    softmax_scale, block_table, lse=None, workspace=None):
    """``flash_attn_varlen_func``'s paged, causal call shape: route by ``max_query_len``."""
    if max_query_len <= 1:
        return paged_decode(q, key_cache, value_cache, block_table, seq_lens, softmax_scale, out,
                            lse=lse, query_start_loc=query_start_loc, workspace=workspace)
    return chunked_prefill(q, key_cache, value_cache, block_table, seq_lens, query_start_loc,
                           softmax_scale, out, lse=lse)
