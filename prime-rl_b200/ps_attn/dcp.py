"""Decode context parallelism (DCP): one sequence's KV spread over the GPUs of
a group, for long contexts with few KV heads.

vLLM's placement (``vllm/v1/worker/block_table.py:326-380``,
``cp_kv_cache_interleave_size``): position ``p`` of a sequence is stored by
rank ``(p // I) % world`` at local index ``(p // (world*I)) * I + p % I`` of
that rank's paged cache, through a block table every rank shares.  Each rank
holds ``hq_local`` query heads; the group attends with the ``world *
hq_local`` heads in rank order and every rank keeps its own heads' output.

One :func:`dcp_decode` per rank and layer replaces vLLM's
``FlashAttentionImpl._forward_with_dcp`` (``flash_attn.py:885-983``): the
query all_gather, the context attention, ``cp_lse_ag_out_rs``
(``vllm/v1/attention/ops/common.py:195-225``), the new tokens' attention and
``merge_attn_states``, plus the KV append of the new tokens.  The exchanges
run inside the library's kernels over NVLink peer memory (a "slab" per rank,
mapped into the others with CUDA IPC); no NCCL call is made per step.

:class:`DcpComm` is one rank's handle on the group.  Build it with
:meth:`DcpComm.from_process_group` (one process per GPU; the IPC handles are
exchanged once through the process group) or, for a single process that
plays every rank on one GPU, with :meth:`DcpComm.emulated` and run
:func:`dcp_decode_group`.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _lib, peer
from .ops import DecodeWorkspace, _problem, _require_cuda, _stream_ptr


# ------------------------------------------------------------ placement
def local_context_lens(seq_lens: torch.Tensor, world: int, rank: int,
                       interleave: int = 1) -> torch.Tensor:
    """Context tokens (the new token excluded) each sequence has on ``rank``:
    ``get_dcp_local_seq_lens(seq_lens - 1, world, rank, interleave)``
    (``vllm/v1/attention/backends/utils.py:857-894``)."""
    L = seq_lens.to(torch.int64) - 1
    base = L // interleave // world * interleave
    rem = L - base * world
    return (base + (rem - rank * interleave).clamp(0, interleave)).to(torch.int32)


def owner(positions: torch.Tensor, world: int, interleave: int = 1) -> torch.Tensor:
    """Rank that stores each position."""
    return (positions // interleave) % world


def local_index(positions: torch.Tensor, world: int, interleave: int = 1) -> torch.Tensor:
    """Index of each position among its owner's tokens of the sequence."""
    return (positions // (world * interleave)) * interleave + positions % interleave


def local_slots(positions: torch.Tensor, block_table_rows: torch.Tensor, block_size: int,
                world: int, rank: int, interleave: int = 1) -> torch.Tensor:
    """Slot of each (sequence row, position) in ``rank``'s cache, -1 where
    another rank stores it: vLLM's ``_compute_slot_mapping_kernel``.
    ``block_table_rows`` [T, P] is the block-table row of each position."""
    pos = positions.to(torch.int64)
    j = local_index(pos, world, interleave)
    blk = torch.gather(block_table_rows.to(torch.int64), 1, (j // block_size)[:, None])[:, 0]
    slot = blk * block_size + j % block_size
    return torch.where(owner(pos, world, interleave) == rank, slot, torch.full_like(slot, -1))


def shard_sequence_kv(keys: list, values: list, block_table: torch.Tensor, key_caches: list,
                      value_caches: list, interleave: int = 1) -> None:
    """Write whole sequences into every rank's cache by the placement rule.

    keys/values: per sequence ``[L_b, Hkv, D]`` tensors (positions 0..L_b-1);
    key_caches/value_caches: per rank ``[NB, bs, Hkv, D]`` (written in place).
    """
    world = len(key_caches)
    bs = key_caches[0].shape[1]
    for b, (k, v) in enumerate(zip(keys, values)):
        pos = torch.arange(k.shape[0], device=k.device)
        own = owner(pos, world, interleave)
        j = local_index(pos, world, interleave)
        row = block_table[b].to(k.device).to(torch.int64)
        for r in range(world):
            sel = own == r
            jr = j[sel]
            blk, off = row[jr // bs], jr % bs
            key_caches[r][blk, off] = k[sel].to(key_caches[r].device)
            value_caches[r][blk, off] = v[sel].to(value_caches[r].device)


# ------------------------------------------------------------ the group
def exchange_handles(handle: bytes, group=None) -> list:
    """All ranks' 64-byte slab handles, in rank order (one all_gather_object)."""
    return peer.exchange_handles(handle, group)


@dataclass
class DcpComm:
    """One rank's view of a DCP group: its slab and every rank's slab address."""

    interleave: int
    max_tokens: int
    hq_local: int
    peers: peer.PeerSlabs

    @property
    def world(self) -> int:
        return self.peers.world

    @property
    def rank(self) -> int:
        return self.peers.rank

    @property
    def slabs(self) -> list:
        return self.peers.slabs

    @property
    def device(self) -> torch.device:
        return self.peers.device

    @staticmethod
    def slab_bytes(max_tokens: int, hq_local: int, world: int) -> int:
        n = _lib.load().ps_dcp_slab_bytes(max_tokens, hq_local, world)
        if n < 0:
            _lib.check(_lib.PS_ERR_INVALID_ARGUMENT)
        return int(n)

    @classmethod
    def from_process_group(cls, max_tokens: int, hq_local: int, interleave: int = 1,
                           group=None, device=None) -> "DcpComm":
        """Collective over ``group`` (one rank per GPU): allocate this rank's
        slab on ``device`` and map every peer's."""
        import torch.distributed as dist

        world = dist.get_world_size(group)
        if world > _lib.PS_DCP_MAX_WORLD:
            raise ValueError(f"DCP groups have at most {_lib.PS_DCP_MAX_WORLD} ranks")
        slabs = peer.PeerSlabs.from_process_group(cls.slab_bytes(max_tokens, hq_local, world),
                                                  group, device)
        return cls(interleave, max_tokens, hq_local, slabs)

    @classmethod
    def emulated(cls, world: int, max_tokens: int, hq_local: int, interleave: int = 1,
                 device=None) -> list:
        """``world`` ranks of a group on one GPU (one process): every slab is
        local.  Use with :func:`dcp_decode_group`."""
        views = peer.PeerSlabs.emulated(world, cls.slab_bytes(max_tokens, hq_local, world), device)
        return [cls(interleave, max_tokens, hq_local, v) for v in views]

    def close(self) -> None:
        self.peers.close()

    def workspace(self, max_num_seqs: int, num_kv_heads: int, head_size: int = 128) -> DecodeWorkspace:
        """A decode workspace sized for the group's heads."""
        return DecodeWorkspace(max_num_seqs, self.hq_local * self.world, num_kv_heads, head_size,
                               self.device)


# ------------------------------------------------------------ the step
def _dcp_problem(comm: DcpComm, q, key_cache, value_cache, block_table, seq_lens, softmax_scale,
                 out, new_key, new_value, slot_mapping, lse) -> _lib.DcpProblem:
    _require_cuda(new_key, new_value, slot_mapping)
    T = q.shape[0]
    if q.shape[1] != comm.hq_local:
        raise ValueError(f"q has {q.shape[1]} heads, the group was built for {comm.hq_local}")
    if seq_lens.shape[0] != T:
        raise ValueError("DCP decode takes one query row per sequence")
    if T > comm.max_tokens:
        raise ValueError(f"{T} tokens > the slabs' {comm.max_tokens}")
    if slot_mapping.dtype != torch.int64 or not slot_mapping.is_contiguous() or slot_mapping.shape[0] < T:
        raise ValueError("slot_mapping must be contiguous int64 with a slot per token")
    hkv, d = key_cache.shape[2], key_cache.shape[3]
    for t in (new_key, new_value):
        if t.dtype != q.dtype or t.shape[0] < T or t.shape[1:] != (hkv, d) or t.stride(-1) != 1:
            raise ValueError("new key/value must be [T, num_kv_heads, head_size] in the cache dtype")
    dp = _lib.DcpProblem()
    dp.local = _problem(q, key_cache, value_cache, block_table, seq_lens, None, softmax_scale, out, lse)
    dp.local.new_key = new_key.data_ptr()
    dp.local.new_key_stride_token, dp.local.new_key_stride_head = new_key.stride(0), new_key.stride(1)
    dp.local.new_value = new_value.data_ptr()
    dp.local.new_value_stride_token, dp.local.new_value_stride_head = new_value.stride(0), new_value.stride(1)
    dp.local.slot_mapping = slot_mapping.data_ptr()
    dp.world, dp.rank, dp.interleave, dp.max_tokens = comm.world, comm.rank, comm.interleave, comm.max_tokens
    for r, s in enumerate(comm.slabs):
        dp.slabs[r] = s
    return dp


def dcp_decode(comm: DcpComm, q: torch.Tensor, key_cache: torch.Tensor, value_cache: torch.Tensor,
               block_table: torch.Tensor, seq_lens: torch.Tensor, softmax_scale: float,
               out: torch.Tensor, new_key: torch.Tensor, new_value: torch.Tensor,
               slot_mapping: torch.Tensor, workspace: DecodeWorkspace,
               lse: torch.Tensor | None = None) -> torch.Tensor:
    """One DCP decode step on this rank; every rank of the group makes the
    same call (same T, same layer order) on its own GPU.

    q/out [T, hq_local, D]; key_cache/value_cache: this rank's cache;
    block_table [T, P] (shared); seq_lens [T] global lengths with the new
    token; new_key/new_value [T, Hkv, D]; slot_mapping [T] this rank's slots
    (-1 where another rank stores the token, :func:`local_slots`); lse
    [hq_local, T] or None.  The workspace must hold ``world * hq_local`` heads
    (:meth:`DcpComm.workspace`).
    """
    lib = _lib.load()
    dp = _dcp_problem(comm, q, key_cache, value_cache, block_table, seq_lens, softmax_scale, out,
                      new_key, new_value, slot_mapping, lse)
    _lib.check(lib.ps_dcp_decode(ctypes.byref(dp), workspace.buffer.data_ptr(), workspace.nbytes,
                                 _stream_ptr(q.device)))
    return out


def dcp_decode_group(comms: list, calls: list, workspaces: list) -> None:
    """Every rank of an emulated group (:meth:`DcpComm.emulated`) in turn, on
    one GPU: phase k of the step for every rank before phase k+1 for any, so
    no barrier wait starts before its signals.  ``calls[r]`` holds rank r's
    :func:`dcp_decode` keyword arguments (without comm and workspace)."""
    lib = _lib.load()
    probs = []
    for c, kw in zip(comms, calls):
        probs.append(_dcp_problem(c, kw["q"], kw["key_cache"], kw["value_cache"], kw["block_table"],
                                  kw["seq_lens"], kw["softmax_scale"], kw["out"], kw["new_key"],
                                  kw["new_value"], kw["slot_mapping"], kw.get("lse")))
    stream = _stream_ptr(comms[0].device)
    for phase in range(5):
        for dp, ws in zip(probs, workspaces):
            _lib.check(lib.ps_dcp_decode_phase(ctypes.byref(dp), phase, ws.buffer.data_ptr(),
                                               ws.nbytes, stream))
