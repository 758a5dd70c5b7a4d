"""vLLM attention backend over libps_attn.so: the drop-in boundary.

Replaces the FlashAttention backend (``vllm/v1/attention/backends/flash_attn.py``)
for the decoder path prime-rl's inference server runs.  It keeps the
FlashAttention surface:

* KV cache ``[2, num_blocks, block_size, num_kv_heads, head_size]`` with the NHD
  stride order (``flash_attn.py:140-171``);
* KV update: the FlashAttention backend has vLLM call ``do_kv_cache_update``
  (``flash_attn.py:850-883``) before ``forward`` (``flash_attn.py:667-848``).
  This backend sets ``forward_includes_kv_cache_update = True`` and does the
  append inside :meth:`PSAttentionImpl.forward`: decode tokens in the same
  launch as their attention, prefill tokens through the append kernel.
  ``do_kv_cache_update`` keeps FlashAttention's contract for callers that use
  it directly.  ``forward`` writes into the preallocated ``output`` in place;
* metadata built from ``CommonAttentionMetadata`` (``backend.py:353-379``):
  ``query_start_loc``, ``seq_lens``, ``block_table``, ``slot_mapping``.

Register it as the CUSTOM backend (select with ``--attention-backend CUSTOM``)
or as an override of FLASH_ATTN::

    from ps_attn.backend import register
    register()                      # CUSTOM
    register(override_flash=True)   # FLASH_ATTN -> PS
    register(rope_fusion=True)      # variant with the fused RoPE + KV append

The ``rope_fusion`` variant (:class:`PSRopeAttentionBackend`) keeps
FlashAttention's ``forward_includes_kv_cache_update = False``, so vLLM issues
the KV update itself and its RoPE + KV-cache fusion pass
(``vllm/compilation/passes/fusion/rope_kvcache_fusion.py``) can replace
``rotary_embedding`` + ``unified_kv_cache_update`` by
:meth:`PSRopeAttentionImpl.do_rope_and_kv_cache_update` (``ps_rope_kv_append``);
its forward does not append.

Batches are reordered decode-first (``reorder_batch_threshold = 1``); decode
requests run the split-KV decode kernel, the rest the chunked-prefill kernel.
With ``PS_ATTN_CASCADE=1`` the metadata builder also finds groups of decode
requests that share their leading KV pages (GRPO samples of one prompt; vLLM
itself only uses cascade attention when every request shares one prefix,
``flash_attn.py:1088-1130``) once per step, and the decode reads each shared
prefix once per group pass.
An fp8 KV cache (``kv_cache_dtype`` "fp8" / "fp8_e4m3", per-tensor scales
``layer._k_scale`` / ``layer._v_scale``) is stored as e4m3(x / scale) by the
append (bit-identical to ``reshape_and_cache_flash`` with "fp8") and read by
the decode kernel's fp8 mode; prefill requests attend over their pages
copied into a 16-bit scratch (``ops.dequant_gather``: the e4m3 values are
exact in bf16) and attended with the scales applied in the prefill kernel.
Unsupported options (ALiBi, sliding window, soft-cap, sinks, other KV-cache
dtypes, encoder attention) raise ``NotImplementedError`` at construction.
"""
from __future__ import annotations

import os
from dataclasses import dataclass
from typing import ClassVar

import torch

from vllm.v1.attention.backend import (AttentionBackend, AttentionCGSupport, AttentionImpl,
                                       AttentionMetadataBuilder, AttentionType,
                                       CommonAttentionMetadata, MultipleOf)
from vllm.v1.attention.backends.utils import split_decodes_and_prefills

from . import _lib, ops

BACKEND_NAME = "CUSTOM"


class PSAttentionBackend(AttentionBackend):
    supported_dtypes: ClassVar[list[torch.dtype]] = [torch.float16, torch.bfloat16]
    supported_kv_cache_dtypes: ClassVar[list[str]] = ["auto", "float16", "bfloat16", "fp8", "fp8_e4m3"]
    forward_includes_kv_cache_update: bool = True

    @staticmethod
    def get_supported_kernel_block_sizes() -> list[int | MultipleOf]:
        return [MultipleOf(16)]

    @staticmethod
    def get_name() -> str:
        return BACKEND_NAME

    @staticmethod
    def get_impl_cls() -> type["PSAttentionImpl"]:
        return PSAttentionImpl

    @staticmethod
    def get_builder_cls() -> type["PSAttentionMetadataBuilder"]:
        return PSAttentionMetadataBuilder

    @staticmethod
    def get_kv_cache_shape(num_blocks: int, block_size: int, num_kv_heads: int, head_size: int,
                           cache_dtype_str: str = "auto") -> tuple[int, ...]:
        if block_size % 16 != 0:
            raise ValueError("Block size must be a multiple of 16.")
        return (2, num_blocks, block_size, num_kv_heads, head_size)

    @staticmethod
    def get_kv_cache_stride_order(include_num_layers_dimension: bool = False) -> tuple[int, ...]:
        if include_num_layers_dimension:
            # (num_blocks, num_layers, 2, block_size, num_kv_heads, head_size)
            return (2, 0, 1, 3, 4, 5)
        return (0, 1, 2, 3, 4)

    @classmethod
    def supports_head_size(cls, head_size: int) -> bool:
        return head_size == 128

    @classmethod
    def supports_attn_type(cls, attn_type: str) -> bool:
        return attn_type == AttentionType.DECODER

    @classmethod
    def supports_non_causal(cls) -> bool:
        return False

    @classmethod
    def supports_sink(cls) -> bool:
        return False

    @classmethod
    def supports_compute_capability(cls, capability) -> bool:
        return (capability.major, capability.minor) == (10, 0)


@dataclass
class PSAttentionMetadata:
    num_actual_tokens: int
    max_query_len: int
    query_start_loc: torch.Tensor   # int32 [B+1]
    max_seq_len: int
    seq_lens: torch.Tensor          # int32 [B]
    block_table: torch.Tensor       # int32 [B, P]
    slot_mapping: torch.Tensor      # int64 [T]
    num_decodes: int
    num_decode_tokens: int
    num_prefills: int
    workspace: ops.DecodeWorkspace
    causal: bool = True
    cascade_plan: ops.CascadePlan | None = None  # shared-prefix plan of the decode rows
    dcp_comm: object | None = None               # decode context parallel group (ps_attn.dcp.DcpComm)


class PSAttentionMetadataBuilder(AttentionMetadataBuilder[PSAttentionMetadata]):
    # decode batches (q_len 1) replay in full CUDA graphs: fixed-size workspace,
    # no allocation and no host synchronisation inside the kernels
    _cudagraph_support: ClassVar[AttentionCGSupport] = AttentionCGSupport.UNIFORM_SINGLE_TOKEN_DECODE
    reorder_batch_threshold: int | None = 1
    supports_update_block_table: bool = True

    def __init__(self, kv_cache_spec, layer_names, vllm_config, device):
        super().__init__(kv_cache_spec, layer_names, vllm_config, device)
        mc, pc = vllm_config.model_config, vllm_config.parallel_config
        self.num_heads_q = mc.get_num_attention_heads(pc)
        self.num_heads_kv = mc.get_num_kv_heads(pc)
        self.head_size = mc.get_head_size()
        max_seqs = max(vllm_config.scheduler_config.max_num_seqs,
                       vllm_config.compilation_config.max_cudagraph_capture_size or 0)
        self.block_size = kv_cache_spec.block_size
        self.cascade = (cascade_enabled() and max_seqs <= ops.CASCADE_MAX_SEQS
                        and self.num_heads_q // self.num_heads_kv <= 8)
        self.dcp_comm = None
        if getattr(pc, "decode_context_parallel_size", 1) > 1:
            # decode context parallelism: one peer-memory slab per rank of the
            # DCP group, mapped once here (collective over the group, before any
            # graph capture); rows of both decode and prefill steps go through it
            from vllm.distributed.parallel_state import get_dcp_group

            from . import dcp

            self.cascade = False
            # one call carries at most PS_DCP_MAX_TOKENS rows; dcp_decode and
            # dcp_prefill run larger steps in pieces of the slabs' rows
            rows = min(max(max_seqs, vllm_config.scheduler_config.max_num_batched_tokens),
                       _lib.PS_DCP_MAX_TOKENS)
            self.dcp_comm = dcp.DcpComm.from_process_group(
                rows, self.num_heads_q, getattr(pc, "cp_kv_cache_interleave_size", 1),
                group=get_dcp_group().cpu_group, device=device)
            self.workspace = self.dcp_comm.workspace(rows, self.num_heads_kv, self.head_size)
        else:
            self.workspace = ops.DecodeWorkspace(max_seqs, self.num_heads_q, self.num_heads_kv,
                                                 self.head_size, device, cascade=self.cascade)
        self.plan = ops.CascadePlan(max_seqs, device) if self.cascade else None

    def build(self, common_prefix_len: int, common_attn_metadata: CommonAttentionMetadata,
              fast_build: bool = False) -> PSAttentionMetadata:
        m = common_attn_metadata
        if common_prefix_len > 0:
            raise NotImplementedError("cascade attention is not used by the PS backend")
        if not m.causal:
            raise NotImplementedError("the PS backend is causal-only")
        nd, npf, ndt, _ = split_decodes_and_prefills(m, decode_threshold=1)
        plan = None
        if getattr(self, "cascade", False) and nd > 0:
            # once per step, from exactly the arrays forward() hands the decode
            plan = ops.cascade_plan(m.block_table_tensor[:nd], m.seq_lens[:nd], self.num_heads_q,
                                    self.num_heads_kv, self.block_size,
                                    query_start_loc=m.query_start_loc[:nd + 1], plan=self.plan)
        return PSAttentionMetadata(
            num_actual_tokens=m.num_actual_tokens, max_query_len=m.max_query_len,
            query_start_loc=m.query_start_loc, max_seq_len=m.max_seq_len, seq_lens=m.seq_lens,
            block_table=m.block_table_tensor, slot_mapping=m.slot_mapping, num_decodes=nd,
            num_decode_tokens=ndt, num_prefills=npf, workspace=self.workspace, causal=True,
            cascade_plan=plan, dcp_comm=getattr(self, "dcp_comm", None))

    def update_block_table(self, metadata: PSAttentionMetadata, blk_table: torch.Tensor,
                           slot_mapping: torch.Tensor) -> PSAttentionMetadata:
        import copy

        new = copy.copy(metadata)
        new.block_table = blk_table
        new.slot_mapping = slot_mapping
        return new

    def use_cascade_attention(self, *args, **kwargs) -> bool:
        return False


class PSAttentionImpl(AttentionImpl):
    can_return_lse_for_decode: bool = True
    # forward appends the step's keys and values (the backend declares
    # forward_includes_kv_cache_update = True)
    appends_in_forward: bool = True

    def __init__(self, num_heads: int, head_size: int, scale: float, num_kv_heads: int,
                 alibi_slopes: list[float] | None, sliding_window: int | None,
                 kv_cache_dtype: str, logits_soft_cap: float | None = None,
                 attn_type: str = AttentionType.DECODER,
                 kv_sharing_target_layer_name: str | None = None,
                 sinks: torch.Tensor | None = None) -> None:
        if alibi_slopes is not None:
            raise NotImplementedError("ALiBi is not supported by the PS backend")
        if sliding_window is not None:
            raise NotImplementedError("sliding window is not supported by the PS backend")
        if logits_soft_cap:
            raise NotImplementedError("logits soft-cap is not supported by the PS backend")
        if sinks is not None:
            raise NotImplementedError("attention sinks are not supported by the PS backend")
        if kv_cache_dtype not in ("auto", "float16", "bfloat16", "fp8", "fp8_e4m3"):
            raise NotImplementedError(f"kv_cache_dtype {kv_cache_dtype} not supported")
        if attn_type != AttentionType.DECODER:
            raise NotImplementedError("the PS backend implements decoder attention only")
        if head_size != 128:
            raise NotImplementedError(f"head_size {head_size} not supported (128)")
        # vLLM's AttentionImpl.__new__ reads the DCP group size.  Under decode
        # context parallelism vLLM hands the whole batch to forward
        # (flash_attn.py:776-789): decode rows go through dcp.dcp_decode,
        # prefill chunks through dcp.dcp_prefill (the group's slabs are set up
        # by the metadata builder).
        self.dcp = getattr(self, "dcp_world_size", 1) > 1
        if self.dcp and kv_cache_dtype not in ("auto", "float16", "bfloat16"):
            raise NotImplementedError("decode context parallelism over an fp8 cache is not supported")
        self.num_heads = num_heads
        self.head_size = head_size
        self.scale = float(scale)
        self.num_kv_heads = num_kv_heads
        self.kv_cache_dtype = kv_cache_dtype
        self.fp8 = kv_cache_dtype in ("fp8", "fp8_e4m3")
        self.kv_sharing_target_layer_name = kv_sharing_target_layer_name
        self.attn_type = attn_type
        self.num_queries_per_kv = num_heads // num_kv_heads

    def _scales(self, layer) -> dict:
        """The layer's fp8 dequantization scales (vLLM's ``_k_scale`` /
        ``_v_scale``), none for a 16-bit cache."""
        if not self.fp8:
            return {}
        return dict(k_scale=getattr(layer, "_k_scale", None), v_scale=getattr(layer, "_v_scale", None))

    def do_kv_cache_update(self, layer, key: torch.Tensor, value: torch.Tensor,
                           kv_cache: torch.Tensor, slot_mapping: torch.Tensor) -> None:
        key_cache, value_cache = kv_cache.unbind(0)
        ops.kv_append(key, value, key_cache, value_cache, slot_mapping, **self._scales(layer))

    def forward(self, layer, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                kv_cache: torch.Tensor, attn_metadata: PSAttentionMetadata, output: torch.Tensor,
                output_scale: torch.Tensor | None = None,
                output_block_scale: torch.Tensor | None = None) -> torch.Tensor:
        if output_scale is not None or output_block_scale is not None:
            raise NotImplementedError("fused output quantization is not supported")
        if attn_metadata is None:  # profiling run
            return output.fill_(0)
        m = attn_metadata
        key_cache, value_cache = kv_cache.unbind(0)
        nd, ndt = m.num_decodes, m.num_decode_tokens
        T = m.num_actual_tokens
        if self.dcp:
            return self._forward_dcp(query, key, value, key_cache, value_cache, m, output)
        # key/value are None when this layer shares another layer's cache
        append = (self.appends_in_forward and key is not None and value is not None
                  and self.kv_sharing_target_layer_name is None)
        sc = self._scales(layer)
        if append and T > ndt:  # prefill tokens: into the cache before their attention
            ops.kv_append(key[ndt:T], value[ndt:T], key_cache, value_cache, m.slot_mapping[ndt:T], **sc)
        if nd > 0:
            fused = dict(new_key=key, new_value=value, slot_mapping=m.slot_mapping) if append else {}
            ops.paged_decode(query[:ndt], key_cache, value_cache, m.block_table[:nd],
                             m.seq_lens[:nd], self.scale, output[:ndt],
                             query_start_loc=m.query_start_loc[:nd + 1], workspace=m.workspace,
                             cascade=None if self.fp8 else m.cascade_plan, **fused, **sc)
        if m.num_prefills > 0:
            kc, vc, bt = key_cache, value_cache, m.block_table[nd:]
            if self.fp8:
                # the prefill kernel reads 16-bit pages: the e4m3 values
                # exactly (unscaled), with the scales applied in the kernel
                bs = key_cache.shape[1]
                kc, vc, bt = ops.dequant_gather(key_cache, value_cache, bt, m.seq_lens[nd:],
                                                (m.max_seq_len + bs - 1) // bs, query.dtype)
            ops.chunked_prefill(query[:T], kc, vc, bt, m.seq_lens[nd:], m.query_start_loc[nd:],
                                self.scale, output[:T], workspace=m.workspace, **sc)
        return output


    def _forward_dcp(self, query, key, value, key_cache, value_cache, m, output):
        """Decode context parallelism (``flash_attn.py:885-983``): the cache
        holds this rank's slice of every sequence (vLLM's DCP slot mapping),
        ``seq_lens`` are global; every rank of the group runs the same rows."""
        from . import dcp

        if m.dcp_comm is None:
            raise RuntimeError("DCP metadata without a DCP group (the builder sets it up)")
        if key is None or value is None or self.kv_sharing_target_layer_name is not None:
            raise NotImplementedError("decode context parallelism needs the layer's own key/value")
        nd, ndt, T = m.num_decodes, m.num_decode_tokens, m.num_actual_tokens
        if nd > 0:
            dcp.dcp_decode(m.dcp_comm, query[:ndt], key_cache, value_cache, m.block_table[:nd],
                           m.seq_lens[:nd], self.scale, output[:ndt], key[:ndt], value[:ndt],
                           m.slot_mapping[:ndt], m.workspace)
        if m.num_prefills > 0:
            qsl = m.query_start_loc[nd:] - m.query_start_loc[nd]
            dcp.dcp_prefill(m.dcp_comm, query[ndt:T], key_cache, value_cache, m.block_table[nd:],
                            m.seq_lens[nd:], qsl, m.max_query_len, self.scale, output[ndt:T],
                            key[ndt:T], value[ndt:T], m.slot_mapping[ndt:T], m.workspace)
        return output


class PSRopeAttentionImpl(PSAttentionImpl):
    """Impl for :class:`PSRopeAttentionBackend`: vLLM performs the KV update
    before ``forward`` (``do_kv_cache_update``, or the fused RoPE + update)."""

    appends_in_forward: bool = False

    def fused_rope_kvcache_supported(self) -> bool:
        # the fused kernel stores 16-bit rows; an fp8 cache takes the plain
        # (quantizing) KV update instead
        return not self.fp8

    def do_rope_and_kv_cache_update(self, layer, query: torch.Tensor, key: torch.Tensor,
                                    value: torch.Tensor, positions: torch.Tensor,
                                    cos_sin_cache: torch.Tensor, is_neox: bool,
                                    kv_cache: torch.Tensor,
                                    layer_slot_mapping: torch.Tensor) -> None:
        """``vllm/v1/attention/backend.py:823-841``: RoPE of query and key in
        place, then the KV append of the rotated key (one launch)."""
        key_cache, value_cache = kv_cache.unbind(0)
        ops.rope_kv_append(query, key, value, positions.flatten(), cos_sin_cache, is_neox,
                           key_cache, value_cache, layer_slot_mapping)


class PSRopeAttentionBackend(PSAttentionBackend):
    forward_includes_kv_cache_update: bool = False

    @staticmethod
    def get_impl_cls() -> type["PSRopeAttentionImpl"]:
        return PSRopeAttentionImpl


def cascade_enabled() -> bool:
    """Shared-prefix decode is opt-in (``PS_ATTN_CASCADE=1``)."""
    return os.environ.get("PS_ATTN_CASCADE", "0") == "1"


def register(override_flash: bool = False, rope_fusion: bool = False) -> None:
    """Register the PS backend with vLLM's backend registry (``rope_fusion``:
    the variant whose KV update vLLM issues, fusable with RoPE)."""
    from vllm.v1.attention.backends.registry import AttentionBackendEnum, register_backend

    cls = PSRopeAttentionBackend if rope_fusion else PSAttentionBackend
    target = AttentionBackendEnum.FLASH_ATTN if override_flash else AttentionBackendEnum.CUSTOM
    register_backend(target, f"{cls.__module__}.{cls.__qualname__}")
