"""CPU: decode context parallelism -- the placement and the combine pinned to
vLLM's own code (golden vectors from its Triton kernels), the oracle's DCP
step equal to unsharded attention, the two-rank data flow over gloo, and the
C-ABI's host-side validation."""
from __future__ import annotations

import ctypes
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from dcp_helpers import make_dcp_case
from helpers import GOLDEN, golden_meta
from oracle import ps_oracle
from ps_attn import _lib, dcp

SLOT_CASES = sorted(golden_meta()["dcp"]["slots"])
COMBINE_CASES = sorted(golden_meta()["dcp"]["combine"])


@pytest.mark.parametrize("world,interleave", [(1, 1), (2, 1), (3, 1), (4, 2), (8, 16), (2, 16)])
def test_local_lens_match_vllm(world, interleave):
    from vllm.v1.attention.backends.utils import get_dcp_local_seq_lens

    L = torch.arange(1, 400, dtype=torch.int32)  # global lengths, the new token included
    for r in range(world):
        ref = get_dcp_local_seq_lens(L - 1, world, r, interleave)
        assert torch.equal(dcp.local_context_lens(L, world, r, interleave), ref)
        assert np.array_equal(ps_oracle.dcp_local_lens(L.numpy() - 1, world, r, interleave), ref.numpy())


@pytest.mark.parametrize("name", SLOT_CASES)
def test_placement_matches_vllm_slot_mapping(name):
    d = dict(np.load(GOLDEN / f"dcp_slots_{name}.npz"))
    world, interleave, bs = (int(x) for x in d["shape"])
    qsl, pos, bt = d["query_start_loc"], d["positions"], d["block_table"]
    rows = np.repeat(np.arange(len(qsl) - 1), np.diff(qsl))
    for r in range(world):
        want = d["slots"][r]
        got_o = np.concatenate([ps_oracle.dcp_placement(pos[qsl[b]:qsl[b + 1]], bt[b], bs, world, r, interleave)
                                for b in range(len(qsl) - 1)])
        got_p = dcp.local_slots(torch.from_numpy(pos), torch.from_numpy(bt[rows]), bs, world, r, interleave)
        assert np.array_equal(got_o, want) and np.array_equal(got_p.numpy(), want)
    # every position is stored by exactly one rank
    assert ((d["slots"] >= 0).sum(axis=0) == 1).all()


@pytest.mark.parametrize("name", COMBINE_CASES)
def test_combine_matches_vllm_correct_and_merge(name):
    """vLLM: correct_attn_out per rank, sum over ranks, merge_attn_states."""
    d = dict(np.load(GOLDEN / f"dcp_combine_{name}.npz"))
    out, lse, o_ctx, lse_ctx = ps_oracle.dcp_combine(d["o_r"], np.transpose(d["lse_r"], (0, 2, 1)),
                                                     d["s_out"], d["s_lse"])
    assert np.array_equal(np.isinf(lse_ctx), np.isinf(d["lse_ctx"].T))
    fin = np.isfinite(lse_ctx)
    np.testing.assert_allclose(lse_ctx[fin], d["lse_ctx"].T[fin], rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(lse, d["out_lse"], rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(o_ctx, d["o_ctx"], rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(out, d["out"], rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("world,interleave", [(1, 1), (2, 1), (3, 1), (4, 2), (2, 16)])
def test_oracle_dcp_step_equals_unsharded_attention(world, interleave):
    # lengths 1 (no context) and short ones leave some ranks without tokens
    lens = [1, 2, 3, 17, 40, 129, 300]
    case = make_dcp_case(lens, world, interleave, hq=8 * world, hkv=4, dtype=torch.float32, seed=5)
    want, want_lse = case.expected()
    out, lse = ps_oracle.dcp_decode(case.q_all.numpy(), [c.numpy() for c in case.key_caches],
                                    [c.numpy() for c in case.value_caches], case.block_table.numpy(),
                                    case.seq_lens.numpy(), case.new_key.numpy(), case.new_value.numpy(),
                                    case.softmax_scale, interleave)
    np.testing.assert_allclose(out, want, atol=2e-5)
    np.testing.assert_allclose(lse, want_lse, atol=2e-5)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_worker(rank, world, port, result_q):
    import sys
    from pathlib import Path

    repo = Path(__file__).resolve().parent.parent
    for p in (repo / "prime-rl_b200", repo, repo / "tests"):
        sys.path.insert(0, str(p))
    from dcp_helpers import make_dcp_case
    from oracle import ps_oracle
    from ps_attn import dcp

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        # the slab-handle exchange the GPU group makes once
        handles = dcp.exchange_handles(bytes([rank]) * 64)
        assert handles == [bytes([r]) * 64 for r in range(world)]
        case = make_dcp_case([1, 5, 33, 200], world, 1, hq=8, hkv=2, dtype=torch.float32, seed=9)
        # this rank: attention of the group's heads over its slice
        lens = ps_oracle.dcp_local_lens(case.seq_lens.numpy() - 1, world, rank)
        B = len(lens)
        o, l = ps_oracle.paged_attention(case.q_all.numpy(), case.key_caches[rank].numpy(),
                                         case.value_caches[rank].numpy(), case.block_table.numpy(),
                                         lens, np.arange(B + 1), case.softmax_scale, causal=False)
        # the exchange: every rank's partial output and LSE
        o_all = [torch.empty(o.shape) for _ in range(world)]
        l_all = [torch.empty(l.shape) for _ in range(world)]
        dist.all_gather(o_all, torch.from_numpy(o))
        dist.all_gather(l_all, torch.from_numpy(l))
        h0, h1 = rank * case.hq_local, (rank + 1) * case.hq_local
        g = case.hq // case.hkv
        kk = np.repeat(case.new_key.numpy(), g, axis=1)[:, h0:h1]
        vv = np.repeat(case.new_value.numpy(), g, axis=1)[:, h0:h1]
        s = case.softmax_scale * np.einsum("thd,thd->ht", case.q_all.numpy()[:, h0:h1], kk)
        out, lse, _, _ = ps_oracle.dcp_combine(np.stack([x.numpy()[:, h0:h1] for x in o_all]),
                                               np.stack([x.numpy()[h0:h1] for x in l_all]), vv, s)
        want, want_lse = case.expected()
        np.testing.assert_allclose(out, want[:, h0:h1], atol=2e-5)
        np.testing.assert_allclose(lse, want_lse[h0:h1], atol=2e-5)
        result_q.put((rank, "ok"))
    except Exception as e:  # surface the failure to the parent at once
        result_q.put((rank, repr(e)))
        raise
    finally:
        dist.destroy_process_group()


def test_two_rank_dcp_dataflow_over_gloo():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gloo_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=240) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
    assert results == {0: "ok", 1: "ok"}
    assert all(p.exitcode == 0 for p in procs)


def test_dcp_abi_validates_on_the_host():
    lib = _lib.load()
    assert [f for f, _ in _lib.DcpProblem._fields_] == ["local", "world", "rank", "interleave",
                                                         "max_tokens", "slabs", "flags"]
    assert ctypes.sizeof(_lib.DcpProblem) == ctypes.sizeof(_lib.PagedProblem) + 16 + 8 * 8 + 8
    # slab layout: header, staged q, partials, LSEs, gathered q, local lengths
    T, hl, w = 64, 8, 2
    want = 256 + T * hl * 256 + T * hl * w * 256 + hl * w * T * 4 + T * hl * w * 256 + 256
    assert lib.ps_dcp_slab_bytes(T, hl, w) == want
    assert lib.ps_dcp_slab_bytes(0, hl, w) == -1 and lib.ps_dcp_slab_bytes(T, hl, 9) == -1
    assert lib.ps_dcp_decode(None, None, 0, None) == _lib.PS_ERR_INVALID_ARGUMENT
    dp = _lib.DcpProblem()
    dp.world, dp.rank, dp.interleave, dp.max_tokens = 9, 0, 1, 64
    assert lib.ps_dcp_decode(ctypes.byref(dp), None, 0, None) == _lib.PS_ERR_INVALID_ARGUMENT
    dp.world, dp.rank = 2, 2
    assert lib.ps_dcp_decode(ctypes.byref(dp), None, 0, None) == _lib.PS_ERR_INVALID_ARGUMENT
    dp.rank, dp.local.block_size, dp.interleave = 1, 16, 3
    assert lib.ps_dcp_decode(ctypes.byref(dp), None, 0, None) == _lib.PS_ERR_INVALID_ARGUMENT
    assert b"interleave" in lib.ps_last_error()
    dp.interleave = 4
    assert lib.ps_dcp_decode(ctypes.byref(dp), None, 0, None) == _lib.PS_ERR_INVALID_ARGUMENT
    assert b"slab" in lib.ps_last_error()  # NULL slabs
    dp.slabs[0], dp.slabs[1] = 256, 512
    dp.local.num_seqs, dp.local.num_tokens = 4, 4
    dp.local.query_start_loc = 16
    assert lib.ps_dcp_decode(ctypes.byref(dp), None, 0, None) == _lib.PS_ERR_INVALID_ARGUMENT
    assert b"one query row" in lib.ps_last_error()
    assert lib.ps_dcp_decode_phase(ctypes.byref(dp), 5, None, 0, None) == _lib.PS_ERR_INVALID_ARGUMENT
    dp.flags = 2  # unknown flag
    dp.local.query_start_loc = None
    assert lib.ps_dcp_decode(ctypes.byref(dp), None, 0, None) == _lib.PS_ERR_INVALID_ARGUMENT
    # merge_attn_states: shape and dtype checks on the host
    assert lib.ps_merge_attn_states(None, 0, 0, None, None, 0, 0, None, None, 0, 0, None, 4, 8, 128,
                                    _lib.PS_DTYPE_BF16, None) == _lib.PS_ERR_INVALID_ARGUMENT
    args = [256, 1024, 128, 512, 256, 1024, 128, 512, 256, 1024, 128, None, 4, 8, 128, _lib.PS_DTYPE_FP32, None]
    assert lib.ps_merge_attn_states(*args) == _lib.PS_ERR_UNSUPPORTED
    args[15], args[14] = _lib.PS_DTYPE_BF16, 64
    assert lib.ps_merge_attn_states(*args) == _lib.PS_ERR_UNSUPPORTED


@pytest.mark.parametrize("world,interleave", [(2, 1), (4, 4)])
def test_dcp_workload_places_every_new_token_once(world, interleave):
    """bench.py's per-rank DCP batches: one shared block table, the new
    token of every sequence stored by exactly one rank, at the slot the
    oracle's placement gives; local context lengths add up to the global."""
    from ps_attn import workloads

    batches = [workloads.make_dcp_config(2, world, r, interleave) for r in range(world)]
    bt = batches[0].block_table
    assert all(torch.equal(b.block_table, bt) for b in batches)
    slots = torch.stack([b.slot_mapping for b in batches])  # [world, B]
    assert ((slots >= 0).sum(0) == 1).all()
    lens = batches[0].seq_lens.numpy()
    for r, b in enumerate(batches):
        want = np.array([ps_oracle.dcp_placement([L - 1], bt[i].numpy(), 16, world, r, interleave)[0]
                         for i, L in enumerate(lens)])
        assert np.array_equal(b.slot_mapping.numpy(), want)
    assert sum(b.unique_tokens for b in batches) == int((lens - 1).sum())


def test_bench_rejects_unsupported_mode_combinations():
    import subprocess
    import sys
    from pathlib import Path

    repo = Path(__file__).resolve().parent.parent
    for args in (["--dcp", "--kv-fp8"], ["--dcp", "--config", "4"], ["--kv-fp8", "--config", "4"],
                 ["--kv-fp8", "--cascade", "--config", "3"]):
        r = subprocess.run([sys.executable, str(repo / "bench.py"), *args], capture_output=True,
                           text=True, timeout=120, cwd=repo)
        assert r.returncode == 2 and "error" in r.stderr, (args, r.returncode, r.stderr[-300:])


@pytest.mark.parametrize("world,interleave", [(1, 1), (2, 1), (3, 2), (4, 16)])
def test_oracle_dcp_prefill_equals_causal_attention(world, interleave):
    """vLLM's DCP evaluation of multi-token chunks (context over the ranks'
    slices, non-causal; the chunk causal over itself; merged) equals causal
    attention over the whole sequence.  Contexts of 0 tokens and chunks of 1
    (a decode row) included."""
    import math

    from ps_attn import dcp

    g = torch.Generator().manual_seed(17)
    ctx = [0, 5, 40, 300, 1]
    qlen = [3, 1, 17, 9, 6]
    hq, hkv, D, bs = 8, 2, 128, 16
    B = len(ctx)
    span = world * interleave
    P = max(math.ceil((c + 1) / span) * interleave for c in ctx) // bs + 2
    NB = B * P + 3
    bt = torch.randperm(NB, generator=g)[:B * P].to(torch.int32).view(B, P)
    kcs = [torch.randn(NB, bs, hkv, D, generator=g) for _ in range(world)]  # stale contents
    vcs = [torch.randn(NB, bs, hkv, D, generator=g) for _ in range(world)]
    ctx_k = [torch.randn(c, hkv, D, generator=g) for c in ctx]
    ctx_v = [torch.randn(c, hkv, D, generator=g) for c in ctx]
    dcp.shard_sequence_kv(ctx_k, ctx_v, bt, kcs, vcs, interleave)
    T = sum(qlen)
    qsl = np.concatenate([[0], np.cumsum(qlen)])
    q = torch.randn(T, hq, D, generator=g)
    nk = torch.randn(T, hkv, D, generator=g)
    nv = torch.randn(T, hkv, D, generator=g)
    lens = np.array(ctx) + np.array(qlen)
    scale = 1.0 / math.sqrt(D)
    out, lse = ps_oracle.dcp_prefill(q.numpy(), [c.numpy() for c in kcs], [c.numpy() for c in vcs],
                                     bt.numpy(), lens, qsl, nk.numpy(), nv.numpy(), scale, interleave)
    for b in range(B):
        t0, t1 = qsl[b], qsl[b + 1]
        k = torch.cat([ctx_k[b], nk[t0:t1]]).numpy()
        v = torch.cat([ctx_v[b], nv[t0:t1]]).numpy()
        want, want_lse = ps_oracle.attention_ref(q[t0:t1].numpy(), k, v, causal=True, softmax_scale=scale)
        np.testing.assert_allclose(out[t0:t1], want, atol=2e-5)
        np.testing.assert_allclose(lse[:, t0:t1], want_lse, atol=2e-5)


def test_dcp_decode_runs_large_steps_in_pieces(monkeypatch):
    """More rows than the slabs hold run as consecutive calls over pieces of
    max_tokens rows, each with its rows' slices of every per-row tensor."""
    from types import SimpleNamespace

    from ps_attn import dcp

    seen = []

    def fake_problem(comm, q, kc, vc, bt, sl, scale, out, nk, nv, slots, lse, context_only):
        seen.append((q[:, 0, 0].tolist(), bt[:, 0].tolist(), sl.tolist(), out.data_ptr(),
                     None if nk is None else nk[:, 0, 0].tolist(),
                     None if slots is None else slots.tolist(),
                     None if lse is None else (lse.shape, lse.stride(), lse.data_ptr())))
        return SimpleNamespace()

    class Lib:
        def ps_dcp_decode(self, *a):
            return 0

    monkeypatch.setattr(dcp, "_dcp_problem", fake_problem)
    monkeypatch.setattr(dcp._lib, "load", lambda *a, **k: Lib())
    monkeypatch.setattr(dcp, "_stream_ptr", lambda dev: 0)
    monkeypatch.setattr(dcp.ctypes, "byref", lambda x: x)
    T, hl = 10, 2
    q = torch.arange(T, dtype=torch.float32)[:, None, None].expand(T, hl, 4).contiguous()
    bt = torch.arange(T, dtype=torch.int32)[:, None].expand(T, 3).contiguous()
    sl = torch.arange(100, 100 + T, dtype=torch.int32)
    out = torch.zeros(T, hl, 4)
    nk = q[:, :1].clone()
    slots = torch.arange(T, dtype=torch.int64) * 7
    lse = torch.zeros(hl, T)
    comm = SimpleNamespace(max_tokens=4)
    ws = SimpleNamespace(buffer=torch.zeros(1), nbytes=1)
    dcp.dcp_decode(comm, q, None, None, bt, sl, 1.0, out, nk, nk, slots, ws, lse=lse)
    assert [s[0] for s in seen] == [[0, 1, 2, 3], [4, 5, 6, 7], [8, 9]]
    assert [s[1] for s in seen] == [[0, 1, 2, 3], [4, 5, 6, 7], [8, 9]]
    assert [s[2] for s in seen] == [[100, 101, 102, 103], [104, 105, 106, 107], [108, 109]]
    assert [s[4] for s in seen] == [[0, 1, 2, 3], [4, 5, 6, 7], [8, 9]]
    assert [s[5] for s in seen] == [[0, 7, 14, 21], [28, 35, 42, 49], [56, 63]]
    assert [s[3] for s in seen] == [out[i].data_ptr() for i in (0, 4, 8)]
    # lse pieces: columns of [hl, T] (head stride T, token stride 1)
    assert [s[6] for s in seen] == [((hl, 4), (T, 1), lse[:, 0].data_ptr()),
                                    ((hl, 4), (T, 1), lse[:, 4].data_ptr()),
                                    ((hl, 2), (T, 1), lse[:, 8].data_ptr())]
    seen.clear()
    dcp.dcp_decode(comm, q[:3], None, None, bt[:3], sl[:3], 1.0, out[:3], None, None, None, ws,
                   context_only=True)
    assert len(seen) == 1 and seen[0][0] == [0, 1, 2]


def test_dcp_chunk_scratch_is_bounded_by_the_tokens(monkeypatch):
    """The chunks' own keys/values go to a scratch paged cache of at most
    T / block_size + B + 1 blocks (not B x the longest chunk): each sequence
    gets its own pages at a running offset, every slot lands in its own
    sequence's pages, and the scratch block table names exactly them."""
    from types import SimpleNamespace

    from ps_attn import dcp, ops

    calls = {}
    monkeypatch.setattr(ops, "kv_append", lambda k, v, kc, vc, slots: calls.update(
        append=(k.shape, kc.shape, slots.clone())))
    monkeypatch.setattr(ops, "chunked_prefill", lambda q, kc, vc, bt, lens, qsl, scale, out, lse=None:
                        calls.update(prefill=(bt.clone(), lens.clone(), kc.shape)))
    bs = 16
    qlens = [1, 300, 2, 17, 16]  # one long chunk among short ones
    qsl = torch.tensor([0] + list(torch.tensor(qlens).cumsum(0)), dtype=torch.int32)
    T, B = int(qsl[-1]), len(qlens)
    hkv, world, rank, hl = 2, 2, 1, 4
    q = torch.zeros(T, hl, 8)
    nk = torch.zeros(T, hkv, 8)
    b_of_t, ql, _ = dcp._chunk_rows(torch.tensor(qlens, dtype=torch.int32) + 5, qsl, T)
    comm = SimpleNamespace(world=world, rank=rank)
    dcp._chunk_attention(comm, q, nk, nk, qsl, ql, b_of_t, max(qlens), bs, 1.0, q.clone(), None)
    nblk = calls["append"][1][0]
    assert nblk == T // bs + B + 1 and nblk < B * ((max(qlens) + bs - 1) // bs)
    slots = calls["append"][2]
    bt, lens, _ = calls["prefill"]
    assert lens.tolist() == qlens
    pages = [(x + bs - 1) // bs for x in qlens]
    for b in range(B):
        own = bt[b, :pages[b]].tolist()
        assert own == list(range(sum(pages[:b]), sum(pages[:b]) + pages[b]))
        for i in range(qlens[b]):
            s = int(slots[int(qsl[b]) + i])
            assert s // bs == own[i // bs] and s % bs == i % bs
    assert int(bt.max()) < nblk and int(slots.max()) < nblk * bs
