"""Multi-GPU sharding of paged decode.

Two schemes, one process per GPU (``torch.distributed``; NCCL on GPUs):

* **KV-head sharding** (tensor parallel, as vLLM's TP splits heads in
  ``vllm/model_executor/models/qwen3.py:78-107``): rank r owns KV heads
  ``[r*Hkv/n, (r+1)*Hkv/n)`` and their GQA query heads, holds only those heads
  of the cache (``[2, NB, bs, Hkv/n, D]``), appends and attends locally, and
  the head outputs are all-gathered over NVLink.  Block tables, ``seq_lens``
  and ``slot_mapping`` are replicated.  GQA groups never cross ranks.
* **Sequence-batch sharding** (data parallel): whole sequences per rank, no
  data-path collective.  :func:`balance_sequences` splits a batch by total
  KV length, keeping GRPO groups (shared prefix pages) on one rank.

The attention call is injected (``attend``), so the host logic is the same
whether the per-rank compute is the CUDA kernel or a CPU checker.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

import torch


@dataclass(frozen=True)
class HeadShard:
    world: int
    rank: int
    num_q_heads: int
    num_kv_heads: int

    def __post_init__(self):
        if self.num_kv_heads % self.world:
            raise ValueError(f"{self.num_kv_heads} KV heads do not divide over {self.world} ranks")
        if self.num_q_heads % self.num_kv_heads:
            raise ValueError("num_q_heads must be a multiple of num_kv_heads")

    @property
    def kv_per_rank(self) -> int:
        return self.num_kv_heads // self.world

    @property
    def q_per_rank(self) -> int:
        return self.num_q_heads // self.world

    @property
    def kv_heads(self) -> tuple[int, int]:
        return self.rank * self.kv_per_rank, (self.rank + 1) * self.kv_per_rank

    @property
    def q_heads(self) -> tuple[int, int]:
        return self.rank * self.q_per_rank, (self.rank + 1) * self.q_per_rank

    def shard_cache(self, kv_cache: torch.Tensor) -> torch.Tensor:
        """This rank's heads of a full ``[2, NB, bs, Hkv, D]`` cache (a copy)."""
        h0, h1 = self.kv_heads
        return kv_cache[:, :, :, h0:h1].contiguous()

    def shard_q(self, q: torch.Tensor) -> torch.Tensor:
        h0, h1 = self.q_heads
        return q[:, h0:h1]

    def shard_kv_rows(self, x: torch.Tensor) -> torch.Tensor:
        h0, h1 = self.kv_heads
        return x[:, h0:h1]


class HeadShardedDecode:
    """Per-rank decode + all-gather of head outputs.

    ``attend(q_local, out_local)`` must write ``[T, Hq/n, D]`` into
    ``out_local``.  The local output is written straight into this rank's
    slot of the gather buffer ``[n, T, Hq/n, D]``; one
    ``all_gather_into_tensor`` fills the other slots, and :meth:`run` returns
    the ``[T, Hq, D]`` result (head order = global head index).
    """

    def __init__(self, shard: HeadShard, max_tokens: int, head_size: int, dtype, device,
                 group=None):
        self.shard = shard
        self.group = group
        self.gather_buf = torch.empty(shard.world, max_tokens, shard.q_per_rank, head_size,
                                      dtype=dtype, device=device)

    def local_out(self, num_tokens: int) -> torch.Tensor:
        return self.gather_buf[self.shard.rank, :num_tokens]

    def run(self, attend: Callable[[torch.Tensor], None], num_tokens: int,
            out: torch.Tensor | None = None) -> torch.Tensor:
        import torch.distributed as dist

        T = num_tokens
        buf = self.gather_buf[:, :T]
        attend(self.local_out(T))
        if self.shard.world > 1:
            if T == self.gather_buf.shape[1]:
                # output as the dim-0 concatenation of the ranks' slots
                flat = self.gather_buf.view(-1, *self.gather_buf.shape[2:])
                dist.all_gather_into_tensor(flat, self.gather_buf[self.shard.rank],
                                            group=self.group)
            else:
                parts = list(torch.empty_like(buf).unbind(0))
                dist.all_gather(parts, buf[self.shard.rank].contiguous(), group=self.group)
                buf = torch.stack(parts)
        full = buf.permute(1, 0, 2, 3).reshape(T, self.shard.num_q_heads, -1)
        if out is not None:
            out.copy_(full)
            return out
        return full


class PeerHeadGather:
    """KV-head-sharded decode whose head outputs are exchanged over NVLink
    peer memory instead of NCCL (``ps_head_gather``).

    Each rank's decode writes its rows ``[T, Hq/n, D]`` into its own slab
    (:meth:`decode`, through ``ops.paged_decode(out_address=...)``); one
    :meth:`gather` launch then pulls every rank's rows into ``out[T, Hq, D]``
    at head offset ``r * Hq/n`` -- the all_gather + permute of
    :class:`HeadShardedDecode` in one kernel, with two flag barriers and no
    NCCL call.  Build with :meth:`from_process_group` (one process per GPU)
    or :meth:`emulated` (every rank on one GPU; run :func:`gather_group`).
    """

    def __init__(self, shard: HeadShard, max_tokens: int, dtype, slabs, status: torch.Tensor):
        self.shard = shard
        self.max_tokens = max_tokens
        self.dtype = dtype
        self.slabs = slabs
        self.status = status

    @staticmethod
    def slab_bytes(max_tokens: int, q_per_rank: int) -> int:
        from . import _lib

        n = _lib.load().ps_head_gather_slab_bytes(max_tokens, q_per_rank)
        if n < 0:
            _lib.check(_lib.PS_ERR_INVALID_ARGUMENT)
        return int(n)

    @classmethod
    def from_process_group(cls, shard: HeadShard, max_tokens: int, dtype, group=None, device=None):
        from .peer import PeerSlabs

        slabs = PeerSlabs.from_process_group(cls.slab_bytes(max_tokens, shard.q_per_rank), group, device)
        status = torch.zeros(1, dtype=torch.int32, device=slabs.device)
        return cls(shard, max_tokens, dtype, slabs, status)

    @classmethod
    def emulated(cls, num_q_heads: int, num_kv_heads: int, world: int, max_tokens: int, dtype,
                 device=None) -> list:
        from .peer import PeerSlabs

        views = PeerSlabs.emulated(world, cls.slab_bytes(max_tokens, num_q_heads // world), device)
        return [cls(HeadShard(world, r, num_q_heads, num_kv_heads), max_tokens, dtype, v,
                    torch.zeros(1, dtype=torch.int32, device=v.device)) for r, v in enumerate(views)]

    def rows_address(self) -> int:
        from . import _lib

        return self.slabs.own + _lib.PS_HEAD_GATHER_ROWS_OFFSET

    def decode(self, q_local, key_cache, value_cache, block_table, seq_lens, softmax_scale,
               out: torch.Tensor, **kw) -> None:
        """This rank's decode (its heads) into its slab; ``out`` [T, Hq, D] is
        the gather's destination and supplies dtype and rows."""
        from . import ops

        T = q_local.shape[0]
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens > the slabs' {self.max_tokens}")
        shape_ref = out[:T, :self.shard.q_per_rank]
        ops.paged_decode(q_local, key_cache, value_cache, block_table, seq_lens, softmax_scale,
                         shape_ref, out_address=self.rows_address(), **kw)

    def _problem(self, num_tokens: int, out: torch.Tensor):
        from . import _lib, ops

        if out.dtype != self.dtype or out.stride(-1) != 1 or not out.is_cuda:
            raise ValueError("out must be a CUDA tensor of the gather's dtype, last dim contiguous")
        if out.shape[1] != self.shard.num_q_heads or out.shape[0] < num_tokens:
            raise ValueError(f"out must be [>= {num_tokens}, {self.shard.num_q_heads}, D]")
        hp = _lib.HeadGatherProblem()
        hp.world, hp.rank = self.shard.world, self.shard.rank
        hp.num_tokens, hp.hq_local, hp.max_tokens = num_tokens, self.shard.q_per_rank, self.max_tokens
        hp.dtype = ops._DTYPES[self.dtype]
        for r, a in enumerate(self.slabs.slabs):
            hp.slabs[r] = a
        hp.out = out.data_ptr()
        hp.out_stride_token, hp.out_stride_head = out.stride(0), out.stride(1)
        hp.status = self.status.data_ptr()
        return hp

    def gather(self, num_tokens: int, out: torch.Tensor) -> torch.Tensor:
        """Every rank's rows into ``out[:num_tokens]`` (same call on every rank)."""
        import ctypes

        from . import _lib, ops

        hp = self._problem(num_tokens, out)
        _lib.check(_lib.load().ps_head_gather(ctypes.byref(hp), ops._stream_ptr(out.device)))
        return out

    def close(self) -> None:
        self.slabs.close()


class FusedHeadGather(PeerHeadGather):
    """KV-head-sharded decode with the head all-gather fused into the decode
    launch (``ps_paged_decode_head_gather``): the decode stores every output
    row into each peer's slab over NVLink as it finishes the row, so the
    exchange overlaps the rest of the decode, and the launch ends with the
    group's ``[T, Hq, D]`` output in ``out`` on every rank -- no separate
    gather launch.  Slabs hold the group's rows ``[max_tokens, Hq, D]``.

    Every rank's launch waits for the others', so the ranks must be separate
    GPUs (one process per GPU, :meth:`from_process_group`); there is no
    one-GPU emulation of a whole group.
    """

    @staticmethod
    def slab_bytes(max_tokens: int, num_q_heads: int) -> int:
        from . import _lib

        n = _lib.load().ps_decode_head_gather_slab_bytes(max_tokens, num_q_heads)
        if n < 0:
            _lib.check(_lib.PS_ERR_INVALID_ARGUMENT)
        return int(n)

    @classmethod
    def from_process_group(cls, shard: HeadShard, max_tokens: int, dtype, group=None, device=None):
        from .peer import PeerSlabs

        slabs = PeerSlabs.from_process_group(cls.slab_bytes(max_tokens, shard.num_q_heads), group, device)
        status = torch.zeros(1, dtype=torch.int32, device=slabs.device)
        return cls(shard, max_tokens, dtype, slabs, status)

    @classmethod
    def emulated(cls, *args, **kwargs):
        raise NotImplementedError("the fused gather's ranks wait on one another: one GPU per rank")

    def decode(self, q_local, key_cache, value_cache, block_table, seq_lens, softmax_scale,
               out: torch.Tensor, **kw) -> torch.Tensor:
        """This rank's decode and the exchange: ``out[:T]`` ([>= T, Hq, D])
        holds every rank's heads when the launch completes (same call on
        every rank)."""
        from . import ops

        T = q_local.shape[0]
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens > the slabs' {self.max_tokens}")
        hp = self._problem(T, out)
        ops.paged_decode(q_local, key_cache, value_cache, block_table, seq_lens, softmax_scale,
                         out[:T, :self.shard.q_per_rank], head_gather=hp, **kw)
        return out

    def gather(self, num_tokens: int, out: torch.Tensor) -> torch.Tensor:
        raise RuntimeError("the fused head gather has no separate gather step: decode() does it")


def gather_group(gathers: list, num_tokens: int, outs: list) -> None:
    """The head gather of an emulated group (:meth:`PeerHeadGather.emulated`):
    phase k for every rank before phase k+1 for any."""
    import ctypes

    from . import _lib, ops

    lib = _lib.load()
    probs = [g._problem(num_tokens, o) for g, o in zip(gathers, outs)]
    stream = ops._stream_ptr(outs[0].device)
    for phase in range(3):
        for hp in probs:
            _lib.check(lib.ps_head_gather_phase(ctypes.byref(hp), phase, stream))


def balance_sequences(seq_lens, world: int, group_size: int = 1) -> list[list[int]]:
    """Greedy longest-first assignment of sequences (or GRPO groups of
    ``group_size`` consecutive sequences) to ``world`` ranks by total length."""
    seq_lens = [int(x) for x in seq_lens]
    if len(seq_lens) % group_size:
        raise ValueError("batch is not a whole number of groups")
    groups = [list(range(i, i + group_size)) for i in range(0, len(seq_lens), group_size)]
    weight = [sum(seq_lens[j] for j in g) for g in groups]
    order = sorted(range(len(groups)), key=lambda i: -weight[i])
    loads = [0] * world
    out = [[] for _ in range(world)]
    for gi in order:
        r = min(range(world), key=lambda k: (loads[k], k))
        out[r].extend(groups[gi])
        loads[r] += weight[gi]
    return [sorted(x) for x in out]
