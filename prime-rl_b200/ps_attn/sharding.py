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
