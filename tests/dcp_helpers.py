"""A decode batch laid out for decode context parallelism (DCP), with the
unsharded expectation computed by the oracle's single-sequence attention."""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch

from oracle import ps_oracle
from ps_attn import dcp


@dataclass
class DcpCase:
    world: int
    interleave: int
    hq: int
    hkv: int
    block_size: int
    seq_lens: torch.Tensor          # [B] global, the new token included
    block_table: torch.Tensor       # [B, P] shared by the ranks
    q_all: torch.Tensor             # [B, hq, D]
    new_key: torch.Tensor           # [B, hkv, D]
    new_value: torch.Tensor
    key_caches: list                # per rank [NB, bs, hkv, D]: context only
    value_caches: list
    slots: list                     # per rank [B] int64, -1 where another rank stores
    ctx_keys: list                  # per sequence [L-1, hkv, D]
    ctx_values: list
    softmax_scale: float

    @property
    def hq_local(self) -> int:
        return self.hq // self.world

    def q_local(self, r: int) -> torch.Tensor:
        return self.q_all[:, r * self.hq_local:(r + 1) * self.hq_local]

    def expected(self):
        """(out [B, hq, D], lse [hq, B]) of each query over its whole sequence."""
        B = self.q_all.shape[0]
        out = np.zeros(tuple(self.q_all.shape), np.float32)
        lse = np.zeros((self.hq, B), np.float32)
        for b in range(B):
            k = torch.cat([self.ctx_keys[b], self.new_key[b:b + 1]]).float().numpy()
            v = torch.cat([self.ctx_values[b], self.new_value[b:b + 1]]).float().numpy()
            o, l = ps_oracle.attention_ref(self.q_all[b:b + 1].float().numpy(), k, v, causal=False,
                                           softmax_scale=self.softmax_scale)
            out[b], lse[:, b] = o[0], l[:, 0]
        return out, lse

    def expected_caches(self):
        """Every rank's cache after the step's append (numpy fp32)."""
        kcs, vcs = [], []
        for r in range(self.world):
            kc = self.key_caches[r].float().numpy().copy()
            vc = self.value_caches[r].float().numpy().copy()
            ps_oracle.kv_append(self.new_key.float().numpy(), self.new_value.float().numpy(), kc, vc,
                                self.slots[r].numpy())
            kcs.append(kc)
            vcs.append(vc)
        return kcs, vcs


def make_dcp_case(lens, world, interleave=1, hq=32, hkv=8, block_size=16, dtype=torch.bfloat16,
                  seed=0) -> DcpCase:
    g = torch.Generator().manual_seed(seed)
    B, D = len(lens), 128
    lens = [int(x) for x in lens]
    span = world * interleave
    # pages per sequence on a rank: its share of the whole sequence (the new
    # token's slot included), rounded up
    max_local = max(math.ceil(L / span) * interleave for L in lens)
    P = math.ceil(max_local / block_size) + 1
    NB = B * P + 5
    perm = torch.randperm(NB, generator=g)[:B * P].to(torch.int32)
    block_table = perm.view(B, P).contiguous()
    # stale cache contents: random values (masking must hide them)
    key_caches = [torch.randn(NB, block_size, hkv, D, generator=g).to(dtype) for _ in range(world)]
    value_caches = [torch.randn(NB, block_size, hkv, D, generator=g).to(dtype) for _ in range(world)]
    ctx_keys = [torch.randn(L - 1, hkv, D, generator=g).to(dtype) for L in lens]
    ctx_values = [torch.randn(L - 1, hkv, D, generator=g).to(dtype) for L in lens]
    dcp.shard_sequence_kv(ctx_keys, ctx_values, block_table, key_caches, value_caches, interleave)
    q_all = torch.randn(B, hq, D, generator=g).to(dtype)
    new_key = torch.randn(B, hkv, D, generator=g).to(dtype)
    new_value = torch.randn(B, hkv, D, generator=g).to(dtype)
    seq_lens = torch.tensor(lens, dtype=torch.int32)
    pos = seq_lens.to(torch.int64) - 1
    slots = [dcp.local_slots(pos, block_table, block_size, world, r, interleave) for r in range(world)]
    return DcpCase(world, interleave, hq, hkv, block_size, seq_lens, block_table, q_all, new_key,
                   new_value, key_caches, value_caches, slots, ctx_keys, ctx_values, 1.0 / math.sqrt(D))


def make_dcp_prefill_case(ctx, qlen, world, interleave=1, hq=32, hkv=8, block_size=16,
                          dtype=torch.bfloat16, seed=0):
    """Sequences with ``ctx[b]`` cached tokens (sharded over the ranks) and a
    chunk of ``qlen[b]`` new tokens.  Returns a dict of the pieces and the
    expected output (causal attention over context + chunk)."""
    g = torch.Generator().manual_seed(seed)
    B, D = len(ctx), 128
    lens = [c + q for c, q in zip(ctx, qlen)]
    span = world * interleave
    P = math.ceil(max(math.ceil(L / span) * interleave for L in lens) / block_size) + 1
    NB = B * P + 3
    bt = torch.randperm(NB, generator=g)[:B * P].to(torch.int32).view(B, P)
    kcs = [torch.randn(NB, block_size, hkv, D, generator=g).to(dtype) for _ in range(world)]
    vcs = [torch.randn(NB, block_size, hkv, D, generator=g).to(dtype) for _ in range(world)]
    ck = [torch.randn(c, hkv, D, generator=g).to(dtype) for c in ctx]
    cv = [torch.randn(c, hkv, D, generator=g).to(dtype) for c in ctx]
    dcp.shard_sequence_kv(ck, cv, bt, kcs, vcs, interleave)
    T = sum(qlen)
    qsl = torch.tensor([0] + list(np.cumsum(qlen)), dtype=torch.int32)
    q = torch.randn(T, hq, D, generator=g).to(dtype)
    nk = torch.randn(T, hkv, D, generator=g).to(dtype)
    nv = torch.randn(T, hkv, D, generator=g).to(dtype)
    pos = torch.cat([torch.arange(c, c + n) for c, n in zip(ctx, qlen)]).to(torch.int64)
    rows = torch.repeat_interleave(torch.arange(B), torch.tensor(qlen))
    slots = [dcp.local_slots(pos, bt[rows], block_size, world, r, interleave) for r in range(world)]
    scale = 1.0 / math.sqrt(D)
    want = np.zeros((T, hq, D), np.float32)
    for b in range(B):
        t0, t1 = int(qsl[b]), int(qsl[b + 1])
        k = torch.cat([ck[b], nk[t0:t1]]).float().numpy()
        v = torch.cat([cv[b], nv[t0:t1]]).float().numpy()
        want[t0:t1], _ = ps_oracle.attention_ref(q[t0:t1].float().numpy(), k, v, causal=True,
                                                 softmax_scale=scale)
    kc_ref, vc_ref = [], []
    for r in range(world):
        kr, vr = kcs[r].float().numpy().copy(), vcs[r].float().numpy().copy()
        ps_oracle.kv_append(nk.float().numpy(), nv.float().numpy(), kr, vr, slots[r].numpy())
        kc_ref.append(kr)
        vc_ref.append(vr)
    return dict(q=q, new_key=nk, new_value=nv, block_table=bt, seq_lens=torch.tensor(lens, dtype=torch.int32),
                query_start_loc=qsl, max_query_len=max(qlen), key_caches=kcs, value_caches=vcs,
                slots=slots, scale=scale, want=want, kc_ref=kc_ref, vc_ref=vc_ref, hq=hq, hkv=hkv)
