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
                 out, new_key, new_value, slot_mapping, lse, context_only=False) -> _lib.DcpProblem:
    T = q.shape[0]
    if q.shape[1] != comm.hq_local:
        raise ValueError(f"q has {q.shape[1]} heads, the group was built for {comm.hq_local}")
    if seq_lens.shape[0] != T:
        raise ValueError("DCP decode takes one query row per sequence")
    if T > comm.max_tokens:
        raise ValueError(f"{T} tokens > the slabs' {comm.max_tokens}")
    dp = _lib.DcpProblem()
    dp.local = _problem(q, key_cache, value_cache, block_table, seq_lens, None, softmax_scale, out, lse)
    if context_only:
        dp.flags = _lib.PS_DCP_CONTEXT_ONLY
    else:
        _require_cuda(new_key, new_value, slot_mapping)
        if slot_mapping.dtype != torch.int64 or not slot_mapping.is_contiguous() or slot_mapping.shape[0] < T:
            raise ValueError("slot_mapping must be contiguous int64 with a slot per token")
        hkv, d = key_cache.shape[2], key_cache.shape[3]
        for t in (new_key, new_value):
            if t.dtype != q.dtype or t.shape[0] < T or t.shape[1:] != (hkv, d) or t.stride(-1) != 1:
                raise ValueError("new key/value must be [T, num_kv_heads, head_size] in the cache dtype")
        dp.local.new_key = new_key.data_ptr()
        dp.local.new_key_stride_token, dp.local.new_key_stride_head = new_key.stride(0), new_key.stride(1)
        dp.local.new_value = new_value.data_ptr()
        dp.local.new_value_stride_token, dp.local.new_value_stride_head = new_value.stride(0), new_value.stride(1)
        dp.local.slot_mapping = slot_mapping.data_ptr()
    dp.world, dp.rank, dp.interleave, dp.max_tokens = comm.world, comm.rank, comm.interleave, comm.max_tokens
    for r, a in enumerate(comm.slabs):
        dp.slabs[r] = a
    return dp


def dcp_decode(comm: DcpComm, q: torch.Tensor, key_cache: torch.Tensor, value_cache: torch.Tensor,
               block_table: torch.Tensor, seq_lens: torch.Tensor, softmax_scale: float,
               out: torch.Tensor, new_key: torch.Tensor | None, new_value: torch.Tensor | None,
               slot_mapping: torch.Tensor | None, workspace: DecodeWorkspace,
               lse: torch.Tensor | None = None, context_only: bool = False) -> torch.Tensor:
    """One DCP decode step on this rank; every rank of the group makes the
    same call (same T, same layer order) on its own GPU.

    q/out [T, hq_local, D]; key_cache/value_cache: this rank's cache;
    block_table [T, P] (shared); seq_lens [T] global lengths with the new
    token; new_key/new_value [T, Hkv, D]; slot_mapping [T] this rank's slots
    (-1 where another rank stores the token, :func:`local_slots`); lse
    [hq_local, T] or None.  The workspace must hold ``world * hq_local`` heads
    (:meth:`DcpComm.workspace`).  ``context_only``: stop after the cross-rank
    correction (out/lse = attention over the context alone; new_key,
    new_value and slot_mapping unused) -- the first half of
    :func:`dcp_prefill`.

    More rows than the slabs hold (``comm.max_tokens``) run as consecutive
    calls over pieces of ``comm.max_tokens`` rows; the rows are independent
    sequences, and every rank cuts the same T the same way.
    """
    lib = _lib.load()
    T = q.shape[0]
    step = comm.max_tokens
    for i in range(0, T, step) if T > step else (0,):
        j = min(T, i + step)
        sl = slice(i, j)
        dp = _dcp_problem(comm, q[sl], key_cache, value_cache, block_table[sl], seq_lens[sl],
                          softmax_scale, out[sl],
                          None if new_key is None else new_key[sl],
                          None if new_value is None else new_value[sl],
                          None if slot_mapping is None else slot_mapping[sl],
                          None if lse is None else lse[:, sl], context_only)
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
                                  kw["seq_lens"], kw["softmax_scale"], kw["out"], kw.get("new_key"),
                                  kw.get("new_value"), kw.get("slot_mapping"), kw.get("lse"),
                                  kw.get("context_only", False)))
    stream = _stream_ptr(comms[0].device)
    for phase in range(5):
        for dp, ws in zip(probs, workspaces):
            _lib.check(lib.ps_dcp_decode_phase(ctypes.byref(dp), phase, ws.buffer.data_ptr(),
                                               ws.nbytes, stream))


# ------------------------------------------------------------ multi-token chunks
def _chunk_rows(seq_lens, query_start_loc, num_tokens):
    """One row per chunk token: its sequence and the one-row "sequence"
    length (context + 1) of the context part; the row's block table is its
    sequence's (``block_table[b_of_t]``)."""
    B = seq_lens.shape[0]
    dev = seq_lens.device
    qlens = (query_start_loc[1:] - query_start_loc[:-1]).to(torch.int64)
    b_of_t = torch.repeat_interleave(torch.arange(B, device=dev), qlens, output_size=num_tokens)
    ctx = seq_lens.to(torch.int64) - qlens
    return b_of_t, qlens, (ctx[b_of_t] + 1).to(torch.int32)


def _chunk_attention(comm: DcpComm, q, new_key, new_value, query_start_loc, qlens, b_of_t,
                     max_query_len: int, block_size: int, softmax_scale: float, q_out, q_lse):
    """This rank's query heads over the chunks' own keys/values, causal: the
    chunks' rows of its KV heads appended into a scratch paged cache, then
    the chunked-prefill kernel."""
    from . import ops

    T, hl, d = q.shape
    hkv = new_key.shape[1]
    group = hl * comm.world // hkv
    kv0 = comm.rank * hl // group
    kv1 = (comm.rank * hl + hl - 1) // group + 1
    if hl % (kv1 - kv0):
        raise ValueError("the rank's query heads do not map onto whole KV-head groups")
    B = qlens.shape[0]
    maxp = max(1, (max_query_len + block_size - 1) // block_size)
    dev = q.device
    # sequence b gets ceil(q_b / block_size) scratch blocks at a running
    # offset: at most T / block_size + B blocks in all, whatever the mix of
    # chunk lengths (no host synchronisation: the bound uses T and B only)
    nblk = T // block_size + B + 1
    pages = (qlens + block_size - 1) // block_size
    first = torch.cumsum(pages, 0) - pages
    sk = torch.empty(nblk, block_size, kv1 - kv0, d, dtype=q.dtype, device=dev)
    sv = torch.empty_like(sk)
    # entries past a sequence's own pages are never read; clamped into the pool
    bt = (first[:, None] + torch.arange(maxp, device=dev)[None, :]).clamp_(max=nblk - 1).to(torch.int32)
    pos = torch.arange(T, device=dev) - query_start_loc.to(torch.int64)[b_of_t]
    slots = first[b_of_t] * block_size + pos
    ops.kv_append(new_key[:T, kv0:kv1], new_value[:T, kv0:kv1], sk, sv, slots)
    ops.chunked_prefill(q, sk, sv, bt, qlens.to(torch.int32), query_start_loc, softmax_scale, q_out,
                        lse=q_lse)


def dcp_prefill(comm: DcpComm, q: torch.Tensor, key_cache: torch.Tensor, value_cache: torch.Tensor,
                block_table: torch.Tensor, seq_lens: torch.Tensor, query_start_loc: torch.Tensor,
                max_query_len: int, softmax_scale: float, out: torch.Tensor, new_key: torch.Tensor,
                new_value: torch.Tensor, slot_mapping: torch.Tensor, workspace: DecodeWorkspace,
                lse: torch.Tensor | None = None) -> torch.Tensor:
    """A DCP step over multi-token query chunks on this rank (every rank makes
    the same call), vLLM's ``_forward_with_dcp`` for prefill batches
    (``flash_attn.py:885-983``):

    1. the chunk tokens this rank stores are appended to its cache;
    2. every chunk row attends over its sequence's context -- the tokens
       before the chunk -- across the group (:func:`dcp_decode` with
       ``context_only``, each row a one-row sequence);
    3. the chunk attends causally over its own keys/values (this rank's
       heads; every rank has the chunk's key/value rows);
    4. ``merge_attn_states`` of the two.

    q/out [T, hq_local, D] (rows in ``query_start_loc`` order, T = total
    chunk tokens; the context part runs in pieces of the slabs' max_tokens
    rows); seq_lens [B] global lengths with
    the chunk; new_key/new_value [T, Hkv, D]; slot_mapping [T] this rank's
    slots; workspace sized for T rows and the group's heads.
    """
    from . import ops

    T = q.shape[0]
    b_of_t, qlens, seq_rows = _chunk_rows(seq_lens, query_start_loc, T)
    ops.kv_append(new_key[:T], new_value[:T], key_cache, value_cache, slot_mapping[:T])
    ctx_out = torch.empty_like(out[:T])
    ctx_lse = torch.empty(q.shape[1], T, dtype=torch.float32, device=q.device)
    # the context part in pieces of the slabs' rows (every rank cuts the same
    # T the same way); each piece gathers only its rows' block tables
    step = comm.max_tokens
    for i in range(0, T, step):
        sl = slice(i, min(T, i + step))
        dcp_decode(comm, q[sl], key_cache, value_cache, block_table[b_of_t[sl]], seq_rows[sl],
                   softmax_scale, ctx_out[sl], None, None, None, workspace, lse=ctx_lse[:, sl],
                   context_only=True)
    q_out = torch.empty_like(ctx_out)
    q_lse = torch.empty_like(ctx_lse)
    _chunk_attention(comm, q, new_key, new_value, query_start_loc, qlens, b_of_t, max_query_len,
                     key_cache.shape[1], softmax_scale, q_out, q_lse)
    ops.merge_attn_states(out[:T], ctx_out, ctx_lse, q_out, q_lse, output_lse=lse)
    return out


def dcp_prefill_group(comms: list, calls: list, workspaces: list) -> None:
    """:func:`dcp_prefill` for every rank of an emulated group on one GPU
    (the cross-rank part phase by phase, as :func:`dcp_decode_group`).
    ``calls[r]``: rank r's :func:`dcp_prefill` keyword arguments (without
    comm and workspace)."""
    from . import ops

    staged = []
    for c, kw in zip(comms, calls):
        T = kw["q"].shape[0]
        b_of_t, qlens, seq_rows = _chunk_rows(kw["seq_lens"], kw["query_start_loc"], T)
        bt_rows = kw["block_table"][b_of_t]
        ops.kv_append(kw["new_key"][:T], kw["new_value"][:T], kw["key_cache"], kw["value_cache"],
                      kw["slot_mapping"][:T])
        ctx_out = torch.empty_like(kw["out"][:T])
        ctx_lse = torch.empty(kw["q"].shape[1], T, dtype=torch.float32, device=kw["q"].device)
        staged.append((b_of_t, qlens, ctx_out, ctx_lse, dict(
            q=kw["q"], key_cache=kw["key_cache"], value_cache=kw["value_cache"], block_table=bt_rows,
            seq_lens=seq_rows, softmax_scale=kw["softmax_scale"], out=ctx_out, lse=ctx_lse,
            context_only=True)))
    dcp_decode_group(comms, [st[4] for st in staged], workspaces)
    for c, kw, (b_of_t, qlens, ctx_out, ctx_lse, _) in zip(comms, calls, staged):
        q_out = torch.empty_like(ctx_out)
        q_lse = torch.empty_like(ctx_lse)
        _chunk_attention(c, kw["q"], kw["new_key"], kw["new_value"], kw["query_start_loc"], qlens, b_of_t,
                         kw["max_query_len"], kw["key_cache"].shape[1], kw["softmax_scale"], q_out, q_lse)
        ops.merge_attn_states(kw["out"][:kw["q"].shape[0]], ctx_out, ctx_lse, q_out, q_lse,
                              output_lse=kw.get("lse"))
