"""Seeded synthetic paged-attention batches for the five benchmark configs.

Each config follows its description in the benchmark spec: Qwen3 attention
shapes, block_size 16, q/k/v ~ N(0, 1), block tables drawn from a seeded random
permutation of a pool sized to fit, ``seq_lens`` counting the newly appended
tokens.  Lengths and tables come from a CPU ``torch.Generator`` (so they are
identical on every machine); the cache contents are drawn on the target device.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

BLOCK = 16


@dataclass
class PagedBatch:
    q: torch.Tensor             # [T, Hq, D]
    key: torch.Tensor           # [T, Hkv, D] new rows to append
    value: torch.Tensor         # [T, Hkv, D]
    kv_cache: torch.Tensor      # [2, NB, bs, Hkv, D]
    block_table: torch.Tensor   # int32 [B, P]
    seq_lens: torch.Tensor      # int32 [B], includes the new tokens
    query_start_loc: torch.Tensor  # int32 [B+1]
    slot_mapping: torch.Tensor  # int64 [T]
    max_query_len: int
    max_seq_len: int
    softmax_scale: float
    unique_tokens: int = 0      # distinct cached tokens read (shared prefixes once)
    logical_tokens: int = 0     # cached tokens read, summed over sequences
    meta: dict = field(default_factory=dict)

    @property
    def key_cache(self):
        return self.kv_cache[0]

    @property
    def value_cache(self):
        return self.kv_cache[1]

    @property
    def num_seqs(self):
        return self.seq_lens.shape[0]

    @property
    def num_tokens(self):
        return self.q.shape[0]

    def to(self, device):
        moved = {k: (v.to(device) if isinstance(v, torch.Tensor) else v)
                 for k, v in self.__dict__.items()}
        return PagedBatch(**moved)


def make_batch(q_lens, seq_lens, num_q_heads, num_kv_heads, head_size=128, block_size=BLOCK,
               dtype=torch.bfloat16, seed=0, device="cpu", share_groups=None,
               shared_prefix_tokens=0, pool_slack=16, kv_heads_slice=None):
    """Build a batch.

    q_lens/seq_lens: per-sequence query rows and total tokens (new included).
    share_groups: size of GRPO groups whose members share their first
    ``shared_prefix_tokens`` tokens (identical leading block-table entries).
    kv_heads_slice: (start, stop) to materialise only those KV heads (and
    their GQA query heads) -- the per-GPU shard of a head-sharded run.
    """
    q_lens = [int(x) for x in q_lens]
    seq_lens = [int(x) for x in seq_lens]
    B = len(seq_lens)
    g = torch.Generator().manual_seed(seed)
    pages = [(L + block_size - 1) // block_size for L in seq_lens]
    shared_pages = shared_prefix_tokens // block_size if share_groups else 0
    if share_groups:
        assert shared_prefix_tokens % block_size == 0 and B % share_groups == 0
        ngroups = B // share_groups
        private = [max(0, p - shared_pages) for p in pages]
        unique = ngroups * shared_pages + sum(private)
        uniq_tok = sum(seq_lens) - (share_groups - 1) * ngroups * shared_prefix_tokens
    else:
        unique = sum(pages)
        uniq_tok = sum(seq_lens)
    nb = unique + pool_slack
    perm = torch.randperm(nb, generator=g).to(torch.int32)
    maxp = max(1, max(pages) if pages else 1)
    bt = torch.zeros(B, maxp, dtype=torch.int32)
    cur = 0
    if share_groups:
        for grp in range(B // share_groups):
            pre = perm[cur:cur + shared_pages]
            cur += shared_pages
            for j in range(share_groups):
                b = grp * share_groups + j
                npriv = max(0, pages[b] - shared_pages)
                bt[b, :min(shared_pages, pages[b])] = pre[:min(shared_pages, pages[b])]
                bt[b, shared_pages:shared_pages + npriv] = perm[cur:cur + npriv]
                cur += npriv
    else:
        for b in range(B):
            bt[b, :pages[b]] = perm[cur:cur + pages[b]]
            cur += pages[b]
    qsl = torch.zeros(B + 1, dtype=torch.int32)
    qsl[1:] = torch.cumsum(torch.tensor(q_lens, dtype=torch.int64), 0).to(torch.int32)
    T = int(qsl[-1])
    # slots of the new tokens
    slots = torch.empty(T, dtype=torch.int64)
    for b in range(B):
        ql, L = q_lens[b], seq_lens[b]
        pos = torch.arange(L - ql, L, dtype=torch.int64)
        slots[int(qsl[b]):int(qsl[b + 1])] = bt[b, pos // block_size].to(torch.int64) * block_size + pos % block_size
    h0, h1 = (0, num_kv_heads) if kv_heads_slice is None else kv_heads_slice
    grp = num_q_heads // num_kv_heads
    hkv = h1 - h0
    hq = hkv * grp
    dev = torch.device(device)
    gd = torch.Generator(device=dev).manual_seed(seed + 1 + 1000 * h0)
    kv_cache = torch.randn(2, nb, block_size, hkv, head_size, generator=gd, dtype=dtype, device=dev)
    q = torch.randn(T, hq, head_size, generator=gd, dtype=dtype, device=dev)
    key = torch.randn(T, hkv, head_size, generator=gd, dtype=dtype, device=dev)
    value = torch.randn(T, hkv, head_size, generator=gd, dtype=dtype, device=dev)
    return PagedBatch(
        q=q, key=key, value=value, kv_cache=kv_cache,
        block_table=bt.to(dev), seq_lens=torch.tensor(seq_lens, dtype=torch.int32, device=dev),
        query_start_loc=qsl.to(dev), slot_mapping=slots.to(dev),
        max_query_len=max(q_lens) if q_lens else 0, max_seq_len=max(seq_lens) if seq_lens else 0,
        softmax_scale=1.0 / math.sqrt(head_size), unique_tokens=uniq_tok, logical_tokens=sum(seq_lens),
        meta={"num_q_heads_total": num_q_heads, "num_kv_heads_total": num_kv_heads,
              "kv_heads_slice": (h0, h1)})


def _uniform_ints(g, lo, hi, n):
    return torch.randint(lo, hi + 1, (n,), generator=g).tolist()


def config_lengths(cfg: int, seed: int = 0):
    """(q_lens, seq_lens, shape kwargs) of benchmark config ``cfg`` (1..5)."""
    g = torch.Generator().manual_seed(seed)
    if cfg == 1:
        L = _uniform_ints(g, 64, 512, 4)
        return [1] * 4, L, dict(num_q_heads=16, num_kv_heads=8, dtype=torch.float32)
    if cfg == 2:
        ctx = _uniform_ints(g, 1024, 4096, 64)
        return [1] * 64, [c + 1 for c in ctx], dict(num_q_heads=16, num_kv_heads=8)
    if cfg == 3:
        gen = _uniform_ints(g, 0, 8192, 256)
        return [1] * 256, [1024 + x + 1 for x in gen], dict(
            num_q_heads=32, num_kv_heads=8, share_groups=8, shared_prefix_tokens=1024)
    if cfg == 4:
        dec_ctx = _uniform_ints(g, 512, 8192, 128)
        pre_ctx = _uniform_ints(g, 0, 4096, 8)
        q_lens = [1] * 128 + [2048] * 8
        seq = [c + 1 for c in dec_ctx] + [c + 2048 for c in pre_ctx]
        return q_lens, seq, dict(num_q_heads=32, num_kv_heads=8)
    if cfg == 5:
        u = torch.rand(512, generator=g, dtype=torch.float64)
        ctx = torch.exp(math.log(2048) + u * (math.log(32768) - math.log(2048))).round().long().tolist()
        return [1] * 512, [c + 1 for c in ctx], dict(num_q_heads=64, num_kv_heads=8)
    raise ValueError(f"unknown config {cfg}")


def make_config(cfg: int, device="cpu", seed: int = 0, dtype=None, kv_heads_slice=None,
                max_seqs: int | None = None) -> PagedBatch:
    """Batch for config ``cfg``; ``max_seqs`` keeps a seeded prefix subset."""
    q_lens, seq_lens, kw = config_lengths(cfg, seed)
    if max_seqs is not None:
        q_lens, seq_lens = q_lens[:max_seqs], seq_lens[:max_seqs]
        if kw.get("share_groups"):
            n = max(kw["share_groups"], (max_seqs // kw["share_groups"]) * kw["share_groups"])
            q_lens, seq_lens = q_lens[:n], seq_lens[:n]
    if dtype is not None:
        kw["dtype"] = dtype
    return make_batch(q_lens, seq_lens, device=device, seed=seed, kv_heads_slice=kv_heads_slice, **kw)


def hbm_bytes(batch: PagedBatch, head_size=128, with_append=True, unique=True) -> int:
    """Algorithmic HBM bytes of one append + attention step.

    KV read (sum of seq_lens x Hkv x D x 2 (K, V) x elem; with ``unique`` a
    shared prefix counts once) + Q in + O out + appended rows read and
    written + metadata.
    """
    es = batch.kv_cache.element_size()
    hkv = batch.kv_cache.shape[3]
    tokens = batch.unique_tokens if unique else batch.logical_tokens
    kv = tokens * hkv * head_size * 2 * es
    T = batch.num_tokens
    hq = batch.q.shape[1]
    qo = T * hq * head_size * es * 2
    app = (T * hkv * head_size * 2 * es * 2) if with_append else 0
    meta = batch.block_table.numel() * 4 + batch.seq_lens.numel() * 4 + batch.slot_mapping.numel() * 8
    return int(kv + qo + app + meta)


def make_dcp_config(cfg: int, world: int, rank: int, interleave: int = 1, device="cpu",
                    seed: int = 0, block_size: int = BLOCK) -> PagedBatch:
    """Rank ``rank``'s share of config ``cfg`` under decode context
    parallelism over ``world`` GPUs: every sequence's tokens interleaved over
    the ranks (vLLM's placement), all KV heads on every rank, the query heads
    split in rank order.  The block table (virtual blocks of ``block_size *
    world`` positions) and the new tokens' key/value rows are the same on
    every rank; ``slot_mapping`` is this rank's (-1 where another rank stores
    the token); ``seq_lens`` are the global lengths.  Cache contents are
    synthetic N(0, 1) values."""
    from . import dcp

    q_lens, seq_lens, kw = config_lengths(cfg, seed)
    if any(q != 1 for q in q_lens):
        raise ValueError("decode context parallelism takes decode batches")
    hq, hkv = kw["num_q_heads"], kw["num_kv_heads"]
    if hq % world:
        raise ValueError(f"{hq} query heads do not divide over {world} ranks")
    dtype = kw.get("dtype", torch.bfloat16)
    B = len(seq_lens)
    g = torch.Generator().manual_seed(seed)
    vbs = block_size * world
    pages = [(L + vbs - 1) // vbs for L in seq_lens]
    nb = sum(pages) + 16
    perm = torch.randperm(nb, generator=g).to(torch.int32)
    bt = torch.zeros(B, max(pages), dtype=torch.int32)
    cur = 0
    for b in range(B):
        bt[b, :pages[b]] = perm[cur:cur + pages[b]]
        cur += pages[b]
    lens = torch.tensor(seq_lens, dtype=torch.int32)
    slots = dcp.local_slots(lens.to(torch.int64) - 1, bt, block_size, world, rank, interleave)
    dev = torch.device(device)
    gq = torch.Generator(device=dev).manual_seed(seed + 1)
    q_all = torch.randn(B, hq, 128, generator=gq, dtype=dtype, device=dev)
    key = torch.randn(B, hkv, 128, generator=gq, dtype=dtype, device=dev)
    value = torch.randn(B, hkv, 128, generator=gq, dtype=dtype, device=dev)
    gc = torch.Generator(device=dev).manual_seed(seed + 7 + 1000 * rank)
    kv_cache = torch.randn(2, nb, block_size, hkv, 128, generator=gc, dtype=dtype, device=dev)
    hl = hq // world
    local_tokens = int(dcp.local_context_lens(lens, world, rank, interleave).sum())
    return PagedBatch(
        q=q_all[:, rank * hl:(rank + 1) * hl].contiguous(), key=key, value=value, kv_cache=kv_cache,
        block_table=bt.to(dev), seq_lens=lens.to(dev),
        query_start_loc=torch.arange(B + 1, dtype=torch.int32, device=dev), slot_mapping=slots.to(dev),
        max_query_len=1, max_seq_len=max(seq_lens), softmax_scale=1.0 / math.sqrt(128),
        unique_tokens=local_tokens, logical_tokens=sum(seq_lens),
        meta={"num_q_heads_total": hq, "num_kv_heads_total": hkv, "dcp_world": world,
              "dcp_rank": rank, "interleave": interleave})
