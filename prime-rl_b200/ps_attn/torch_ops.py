"""The C ABI as PyTorch operators: ``torch.ops.ps_attn.*``.

Registered with ``torch.library.custom_op`` (mutated arguments declared, so
``torch.compile`` and CUDA-graph capture see the side effects) and a fake
implementation (shape-only, no launch) for tracing:

* ``ps_attn::kv_append(key, value, key_cache!, value_cache!, slot_mapping)`` --
  ``reshape_and_cache_flash`` (``vllm/_custom_ops.py:2591``);
* ``ps_attn::paged_decode(q, key_cache!, value_cache!, block_table, seq_lens,
  query_start_loc?, softmax_scale, max_seq_len, out!, lse!?, workspace!,
  new_key?, new_value?, slot_mapping?)`` -- ``flash_attn_varlen_func`` with
  ``max_seqlen_q == 1`` (``flash_attn.py:796-817``), the decode tokens'
  append fused when ``new_key``/``new_value``/``slot_mapping`` are given
  (the caches are declared mutated for that);
* ``ps_attn::chunked_prefill(q, key_cache, value_cache, block_table,
  seq_lens, query_start_loc, softmax_scale, max_seq_len, out!, lse!?,
  workspace!?)`` -- ``flash_attn_varlen_func`` with ``max_seqlen_q > 1``.

Conventions of the C ABI hold: caller-allocated outputs and workspace (a
``uint8`` tensor of ``DecodeWorkspace``'s size, zeroed once), the current
CUDA stream, no host synchronisation, errors raised as
:class:`ps_attn._lib.PSError`.  ``max_seq_len`` is accepted for signature
parity with vLLM's call and not needed by the kernels.  vLLM's attention
layer already wraps the backend in its own opaque custom op
(``unified_attention_with_output``), so the backend calls :mod:`ps_attn.ops`
directly; these operators serve callers that compose the kernels under
``torch.compile`` themselves.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import ops


class _WorkspaceView:
    """A workspace tensor seen as :class:`ops.DecodeWorkspace` (the library
    checks its size against the call)."""

    def __init__(self, buffer: torch.Tensor, num_seqs: int):
        if buffer.dtype != torch.uint8 or not buffer.is_contiguous():
            raise ValueError("workspace must be a contiguous uint8 tensor")
        self.buffer = buffer
        self.nbytes = buffer.numel()
        self.max_num_seqs = num_seqs


@torch.library.custom_op("ps_attn::kv_append", mutates_args=("key_cache", "value_cache"))
def kv_append(key: torch.Tensor, value: torch.Tensor, key_cache: torch.Tensor, value_cache: torch.Tensor,
              slot_mapping: torch.Tensor) -> None:
    ops.kv_append(key, value, key_cache, value_cache, slot_mapping)


@kv_append.register_fake
def _kv_append_fake(key, value, key_cache, value_cache, slot_mapping) -> None:
    return None


@torch.library.custom_op("ps_attn::paged_decode",
                         mutates_args=("key_cache", "value_cache", "out", "lse", "workspace"))
def paged_decode(q: torch.Tensor, key_cache: torch.Tensor, value_cache: torch.Tensor,
                 block_table: torch.Tensor, seq_lens: torch.Tensor, query_start_loc: Optional[torch.Tensor],
                 softmax_scale: float, max_seq_len: int, out: torch.Tensor, lse: Optional[torch.Tensor],
                 workspace: torch.Tensor, new_key: Optional[torch.Tensor] = None,
                 new_value: Optional[torch.Tensor] = None, slot_mapping: Optional[torch.Tensor] = None) -> None:
    fused = dict(new_key=new_key, new_value=new_value, slot_mapping=slot_mapping) if new_key is not None else {}
    ops.paged_decode(q, key_cache, value_cache, block_table, seq_lens, softmax_scale, out, lse=lse,
                     query_start_loc=query_start_loc,
                     workspace=_WorkspaceView(workspace, seq_lens.shape[0]), **fused)


@paged_decode.register_fake
def _paged_decode_fake(q, key_cache, value_cache, block_table, seq_lens, query_start_loc, softmax_scale,
                       max_seq_len, out, lse, workspace, new_key=None, new_value=None, slot_mapping=None) -> None:
    return None


@torch.library.custom_op("ps_attn::chunked_prefill", mutates_args=("out", "lse", "workspace"))
def chunked_prefill(q: torch.Tensor, key_cache: torch.Tensor, value_cache: torch.Tensor,
                    block_table: torch.Tensor, seq_lens: torch.Tensor, query_start_loc: torch.Tensor,
                    softmax_scale: float, max_seq_len: int, out: torch.Tensor, lse: Optional[torch.Tensor],
                    workspace: Optional[torch.Tensor] = None) -> None:
    ws = None if workspace is None else _WorkspaceView(workspace, seq_lens.shape[0])
    ops.chunked_prefill(q, key_cache, value_cache, block_table, seq_lens, query_start_loc, softmax_scale, out,
                        lse=lse, workspace=ws)


@chunked_prefill.register_fake
def _chunked_prefill_fake(q, key_cache, value_cache, block_table, seq_lens, query_start_loc, softmax_scale,
                          max_seq_len, out, lse, workspace=None) -> None:
    return None


def workspace_tensor(max_num_seqs: int, num_q_heads: int, num_kv_heads: int, head_size: int = 128,
                     device=None) -> torch.Tensor:
    """A zeroed workspace for :func:`paged_decode` / :func:`chunked_prefill`
    (the buffer of an :class:`ops.DecodeWorkspace`)."""
    return ops.DecodeWorkspace(max_num_seqs, num_q_heads, num_kv_heads, head_size, device).buffer
