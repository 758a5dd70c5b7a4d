"""ctypes binding of libps_attn.so (declarations: include/ps_attn.h).

There is no fallback: if the library is missing or fails to load, every op
raises.  ``load()`` builds the library first when its sources are newer.
"""
from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

_LIB = None
_LOCK = threading.Lock()

PS_OK = 0
PS_ERR_INVALID_ARGUMENT = 1
PS_ERR_UNSUPPORTED = 2
PS_ERR_WORKSPACE = 3
PS_ERR_CUDA = 4

PS_DEV_SLOT_OUT_OF_RANGE = 0x1
PS_DEV_BLOCK_OUT_OF_RANGE = 0x2
PS_DEV_WAIT_TIMEOUT = 0x4
PS_DEV_BAD_METADATA = 0x8

PS_DTYPE_FP16 = 0
PS_DTYPE_BF16 = 1
PS_DTYPE_FP32 = 2

PS_KV_AUTO = 0
PS_KV_FP8_E4M3 = 1

ABI_VERSION = 3

# every symbol include/ps_attn.h declares
EXPORTED_SYMBOLS = (
    "ps_abi_version",
    "ps_last_error",
    "ps_kv_append",
    "ps_kv_append_fp8",
    "ps_paged_decode_workspace_size",
    "ps_paged_decode",
    "ps_chunked_prefill",
    "ps_paged_decode_static_scratch",
    "ps_cascade_plan_bytes",
    "ps_cascade_plan_build",
    "ps_paged_decode_cascade_workspace_size",
    "ps_paged_decode_cascade",
    "ps_rope_kv_append",
    "ps_chunked_prefill_ws",
    "ps_dcp_slab_bytes",
    "ps_dcp_slab_alloc",
    "ps_dcp_slab_free",
    "ps_dcp_ipc_handle",
    "ps_dcp_ipc_open",
    "ps_dcp_ipc_close",
    "ps_dcp_decode",
    "ps_dcp_decode_phase",
    "ps_head_gather_slab_bytes",
    "ps_head_gather",
    "ps_head_gather_phase",
    "ps_decode_head_gather_slab_bytes",
    "ps_paged_decode_head_gather",
    "ps_kv_dequant_gather",
    "ps_merge_attn_states",
)
PS_HEAD_GATHER_ROWS_OFFSET = 256

PS_DCP_MAX_WORLD = 8
PS_DCP_IPC_HANDLE_BYTES = 64
# rows of one ps_dcp_decode call (ps_dcp_slab_bytes' max_tokens limit)
PS_DCP_MAX_TOKENS = 4096


class PSError(RuntimeError):
    """A libps_attn call returned a non-zero ps_status."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"ps_attn error {code}: {msg}")
        self.code = code


class PagedProblem(ctypes.Structure):
    """Mirror of ``ps_paged_problem`` in include/ps_attn.h (same field order)."""

    _fields_ = [
        ("q", ctypes.c_void_p),
        ("q_stride_token", ctypes.c_int64),
        ("q_stride_head", ctypes.c_int64),
        ("key_cache", ctypes.c_void_p),
        ("value_cache", ctypes.c_void_p),
        ("cache_stride_block", ctypes.c_int64),
        ("cache_stride_slot", ctypes.c_int64),
        ("cache_stride_head", ctypes.c_int64),
        ("num_blocks", ctypes.c_int64),
        ("block_table", ctypes.c_void_p),
        ("block_table_stride", ctypes.c_int64),
        ("max_blocks_per_seq", ctypes.c_int32),
        ("seq_lens", ctypes.c_void_p),
        ("query_start_loc", ctypes.c_void_p),
        ("num_seqs", ctypes.c_int32),
        ("out", ctypes.c_void_p),
        ("out_stride_token", ctypes.c_int64),
        ("out_stride_head", ctypes.c_int64),
        ("lse", ctypes.c_void_p),
        ("lse_stride_head", ctypes.c_int64),
        ("lse_stride_token", ctypes.c_int64),
        ("num_q_heads", ctypes.c_int32),
        ("num_kv_heads", ctypes.c_int32),
        ("head_size", ctypes.c_int32),
        ("block_size", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("softmax_scale", ctypes.c_float),
        ("num_tokens", ctypes.c_int64),
        ("status", ctypes.c_void_p),
        ("new_key", ctypes.c_void_p),
        ("new_key_stride_token", ctypes.c_int64),
        ("new_key_stride_head", ctypes.c_int64),
        ("new_value", ctypes.c_void_p),
        ("new_value_stride_token", ctypes.c_int64),
        ("new_value_stride_head", ctypes.c_int64),
        ("slot_mapping", ctypes.c_void_p),
        ("kv_cache_dtype", ctypes.c_int32),
        ("k_scale", ctypes.c_void_p),
        ("v_scale", ctypes.c_void_p),
    ]


class RopeAppendProblem(ctypes.Structure):
    """Mirror of ``ps_rope_append_problem`` in include/ps_attn.h (same field order)."""

    _fields_ = [
        ("query", ctypes.c_void_p),
        ("query_stride_token", ctypes.c_int64),
        ("query_stride_head", ctypes.c_int64),
        ("key", ctypes.c_void_p),
        ("key_stride_token", ctypes.c_int64),
        ("key_stride_head", ctypes.c_int64),
        ("value", ctypes.c_void_p),
        ("value_stride_token", ctypes.c_int64),
        ("value_stride_head", ctypes.c_int64),
        ("key_cache", ctypes.c_void_p),
        ("value_cache", ctypes.c_void_p),
        ("cache_stride_block", ctypes.c_int64),
        ("cache_stride_slot", ctypes.c_int64),
        ("cache_stride_head", ctypes.c_int64),
        ("num_blocks", ctypes.c_int64),
        ("block_size", ctypes.c_int32),
        ("slot_mapping", ctypes.c_void_p),
        ("positions", ctypes.c_void_p),
        ("cos_sin_cache", ctypes.c_void_p),
        ("cos_sin_stride", ctypes.c_int64),
        ("max_position", ctypes.c_int64),
        ("cos_sin_dtype", ctypes.c_int32),
        ("rotary_dim", ctypes.c_int32),
        ("is_neox", ctypes.c_int32),
        ("num_tokens", ctypes.c_int64),
        ("num_q_heads", ctypes.c_int32),
        ("num_kv_heads", ctypes.c_int32),
        ("head_size", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("status", ctypes.c_void_p),
    ]


class DcpProblem(ctypes.Structure):
    """Mirror of ``ps_dcp_problem`` in include/ps_attn.h (same field order)."""

    _fields_ = [
        ("local", PagedProblem),
        ("world", ctypes.c_int32),
        ("rank", ctypes.c_int32),
        ("interleave", ctypes.c_int32),
        ("max_tokens", ctypes.c_int32),
        ("slabs", ctypes.c_void_p * PS_DCP_MAX_WORLD),
        ("flags", ctypes.c_int32),
    ]


PS_DCP_CONTEXT_ONLY = 1


class HeadGatherProblem(ctypes.Structure):
    """Mirror of ``ps_head_gather_problem`` in include/ps_attn.h (same field order)."""

    _fields_ = [
        ("world", ctypes.c_int32),
        ("rank", ctypes.c_int32),
        ("num_tokens", ctypes.c_int32),
        ("hq_local", ctypes.c_int32),
        ("max_tokens", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("slabs", ctypes.c_void_p * 8),
        ("out", ctypes.c_void_p),
        ("out_stride_token", ctypes.c_int64),
        ("out_stride_head", ctypes.c_int64),
        ("status", ctypes.c_void_p),
    ]


def lib_path() -> Path:
    """The in-tree library, or a tuning variant named by ``PS_ATTN_LIB``."""
    override = os.environ.get("PS_ATTN_LIB")
    if override:
        return Path(override).resolve()
    return Path(__file__).resolve().parent / "libps_attn.so"


def _declare(lib):
    c = ctypes
    lib.ps_abi_version.restype = c.c_int
    lib.ps_abi_version.argtypes = []
    lib.ps_last_error.restype = c.c_char_p
    lib.ps_last_error.argtypes = []
    lib.ps_kv_append.restype = c.c_int
    lib.ps_kv_append.argtypes = [
        c.c_void_p, c.c_int64, c.c_int64,  # key
        c.c_void_p, c.c_int64, c.c_int64,  # value
        c.c_void_p, c.c_void_p, c.c_int64, c.c_int64, c.c_int64, c.c_int64,  # caches
        c.c_void_p, c.c_int64, c.c_int, c.c_int, c.c_int, c.c_int,  # slots, shape
        c.c_void_p, c.c_void_p,  # status, stream
    ]
    lib.ps_kv_append_fp8.restype = c.c_int
    lib.ps_kv_append_fp8.argtypes = [
        c.c_void_p, c.c_int64, c.c_int64,  # key
        c.c_void_p, c.c_int64, c.c_int64,  # value
        c.c_void_p, c.c_void_p, c.c_int64, c.c_int64, c.c_int64, c.c_int64,  # caches
        c.c_void_p, c.c_int64, c.c_int32, c.c_int32, c.c_int32, c.c_int32,  # slots, shape, dtype
        c.c_void_p, c.c_void_p, c.c_void_p, c.c_void_p,  # scales, status, stream
    ]
    lib.ps_paged_decode_workspace_size.restype = c.c_int64
    lib.ps_paged_decode_workspace_size.argtypes = [c.c_int32] * 4
    lib.ps_paged_decode.restype = c.c_int
    lib.ps_paged_decode.argtypes = [c.POINTER(PagedProblem), c.c_void_p, c.c_int64, c.c_void_p]
    lib.ps_chunked_prefill.restype = c.c_int
    lib.ps_chunked_prefill.argtypes = [c.POINTER(PagedProblem), c.c_void_p]
    lib.ps_paged_decode_static_scratch.restype = c.c_int
    lib.ps_paged_decode_static_scratch.argtypes = [c.POINTER(PagedProblem), c.c_void_p]
    lib.ps_chunked_prefill_ws.restype = c.c_int
    lib.ps_chunked_prefill_ws.argtypes = [c.POINTER(PagedProblem), c.c_void_p, c.c_int64, c.c_void_p]
    lib.ps_rope_kv_append.restype = c.c_int
    lib.ps_rope_kv_append.argtypes = [c.POINTER(RopeAppendProblem), c.c_void_p]
    lib.ps_cascade_plan_bytes.restype = c.c_int64
    lib.ps_cascade_plan_bytes.argtypes = [c.c_int32]
    lib.ps_cascade_plan_build.restype = c.c_int
    lib.ps_cascade_plan_build.argtypes = [c.POINTER(PagedProblem), c.c_int32, c.c_void_p, c.c_int64,
                                          c.c_void_p]
    lib.ps_paged_decode_cascade_workspace_size.restype = c.c_int64
    lib.ps_paged_decode_cascade_workspace_size.argtypes = [c.c_int32] * 4
    lib.ps_paged_decode_cascade.restype = c.c_int
    lib.ps_paged_decode_cascade.argtypes = [c.POINTER(PagedProblem), c.c_void_p, c.c_int64,
                                            c.c_void_p, c.c_int64, c.c_void_p]
    lib.ps_dcp_slab_bytes.restype = c.c_int64
    lib.ps_dcp_slab_bytes.argtypes = [c.c_int32] * 3
    lib.ps_dcp_slab_alloc.restype = c.c_int
    lib.ps_dcp_slab_alloc.argtypes = [c.c_int64, c.POINTER(c.c_void_p)]
    lib.ps_dcp_slab_free.restype = c.c_int
    lib.ps_dcp_slab_free.argtypes = [c.c_void_p]
    lib.ps_dcp_ipc_handle.restype = c.c_int
    lib.ps_dcp_ipc_handle.argtypes = [c.c_void_p, c.c_void_p]
    lib.ps_dcp_ipc_open.restype = c.c_int
    lib.ps_dcp_ipc_open.argtypes = [c.c_void_p, c.POINTER(c.c_void_p)]
    lib.ps_dcp_ipc_close.restype = c.c_int
    lib.ps_dcp_ipc_close.argtypes = [c.c_void_p]
    lib.ps_dcp_decode.restype = c.c_int
    lib.ps_dcp_decode.argtypes = [c.POINTER(DcpProblem), c.c_void_p, c.c_int64, c.c_void_p]
    lib.ps_merge_attn_states.restype = c.c_int
    lib.ps_merge_attn_states.argtypes = [
        c.c_void_p, c.c_int64, c.c_int64, c.c_void_p,  # prefix out, strides, lse
        c.c_void_p, c.c_int64, c.c_int64, c.c_void_p,  # suffix
        c.c_void_p, c.c_int64, c.c_int64, c.c_void_p,  # out, strides, out lse
        c.c_int64, c.c_int32, c.c_int32, c.c_int32, c.c_void_p,
    ]
    lib.ps_kv_dequant_gather.restype = c.c_int
    lib.ps_kv_dequant_gather.argtypes = [c.POINTER(PagedProblem), c.c_int32, c.c_void_p, c.c_void_p,
                                         c.c_void_p]
    lib.ps_head_gather_slab_bytes.restype = c.c_int64
    lib.ps_head_gather_slab_bytes.argtypes = [c.c_int32, c.c_int32]
    lib.ps_head_gather.restype = c.c_int
    lib.ps_head_gather.argtypes = [c.POINTER(HeadGatherProblem), c.c_void_p]
    lib.ps_head_gather_phase.restype = c.c_int
    lib.ps_head_gather_phase.argtypes = [c.POINTER(HeadGatherProblem), c.c_int32, c.c_void_p]
    lib.ps_decode_head_gather_slab_bytes.restype = c.c_int64
    lib.ps_decode_head_gather_slab_bytes.argtypes = [c.c_int32, c.c_int32]
    lib.ps_paged_decode_head_gather.restype = c.c_int
    lib.ps_paged_decode_head_gather.argtypes = [c.POINTER(PagedProblem), c.c_void_p, c.c_int64,
                                                c.POINTER(HeadGatherProblem), c.c_void_p]
    lib.ps_dcp_decode_phase.restype = c.c_int
    lib.ps_dcp_decode_phase.argtypes = [c.POINTER(DcpProblem), c.c_int32, c.c_void_p, c.c_int64,
                                        c.c_void_p]


def load(build_if_stale: bool = True):
    """Load (and, if its sources changed, rebuild) libps_attn.so."""
    global _LIB
    if _LIB is not None:
        return _LIB
    with _LOCK:
        if _LIB is not None:
            return _LIB
        path = lib_path()
        if (build_if_stale and os.environ.get("PS_ATTN_NO_BUILD", "0") != "1"
                and not os.environ.get("PS_ATTN_LIB")):
            from . import _build

            if _build.needs_build():
                try:
                    _build.build()
                except RuntimeError:
                    if not path.exists():
                        raise
        if not path.exists():
            raise RuntimeError(
                f"libps_attn.so not found at {path}; build it with "
                "`python -m ps_attn._build` (needs nvcc)")
        lib = ctypes.CDLL(str(path))
        _declare(lib)
        if lib.ps_abi_version() != ABI_VERSION:
            raise RuntimeError(f"libps_attn ABI {lib.ps_abi_version()} != {ABI_VERSION}")
        _LIB = lib
        return lib


def check(rc: int):
    if rc != PS_OK:
        msg = _LIB.ps_last_error().decode(errors="replace") if _LIB is not None else ""
        raise PSError(rc, msg)
