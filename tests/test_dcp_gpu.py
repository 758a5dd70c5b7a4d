"""GPU: decode context parallelism through the C ABI.

* An emulated group (every rank's slab and cache on one GPU, the ranks run
  phase by phase from one process): each rank's output against the
  unsharded attention (the attention tolerances), the new tokens appended
  bit-exactly where the rank stores them, several steps on the same slabs.
* A bounded barrier wait that runs out (a peer that never signals): the
  status word reports PS_DEV_WAIT_TIMEOUT within about a second.
* With two GPUs present, a real group (one process per GPU, slabs mapped
  over CUDA IPC, the exchanges over NVLink).
"""
from __future__ import annotations

import ctypes
import datetime
import os
import socket
import time

import numpy as np
import pytest
import torch

from dcp_helpers import make_dcp_case
from helpers import assert_attn_close
from ps_attn import _lib, dcp

pytestmark = pytest.mark.gpu


def _rank_call(case, r, dev, out, lse):
    return dict(q=case.q_local(r).to(dev), key_cache=case.key_caches[r].to(dev),
                value_cache=case.value_caches[r].to(dev), block_table=case.block_table.to(dev),
                seq_lens=case.seq_lens.to(dev), softmax_scale=case.softmax_scale, out=out,
                new_key=case.new_key.to(dev), new_value=case.new_value.to(dev),
                slot_mapping=case.slots[r].to(dev), lse=lse)


def _check_rank(case, r, call, want, want_lse, kcs, vcs):
    h0, h1 = r * case.hq_local, (r + 1) * case.hq_local
    assert_attn_close(call["out"].float().cpu().numpy(), want[:, h0:h1],
                      call["lse"].cpu().numpy(), want_lse[h0:h1])
    assert np.array_equal(call["key_cache"].float().cpu().numpy(), kcs[r])
    assert np.array_equal(call["value_cache"].float().cpu().numpy(), vcs[r])


@pytest.mark.parametrize("world,interleave,hq,hkv", [
    (1, 1, 32, 8), (2, 1, 32, 8), (2, 16, 64, 8), (4, 1, 64, 8), (4, 4, 16, 8), (8, 1, 64, 8),
])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_emulated_group_matches_unsharded_attention(cuda_device, world, interleave, hq, hkv, dtype):
    lens = [1, 2, 5, 17, 64, 300, 1025, 4100, 9000, 33]
    T = len(lens)
    comms = dcp.DcpComm.emulated(world, T, hq // world, interleave, cuda_device)
    wss = [c.workspace(T, hkv) for c in comms]
    try:
        for step in range(3):  # the same slabs serve consecutive steps
            case = make_dcp_case(lens, world, interleave, hq, hkv, dtype=dtype, seed=100 + step)
            calls = []
            for r in range(world):
                out = torch.full((T, case.hq_local, 128), float("nan"), dtype=dtype, device=cuda_device)
                lse = torch.empty(case.hq_local, T, dtype=torch.float32, device=cuda_device)
                calls.append(_rank_call(case, r, cuda_device, out, lse))
            dcp.dcp_decode_group(comms, calls, wss)
            torch.cuda.synchronize()
            want, want_lse = case.expected()
            kcs, vcs = case.expected_caches()
            for r in range(world):
                assert wss[r].status() == 0
                _check_rank(case, r, calls[r], want, want_lse, kcs, vcs)
    finally:
        for c in comms:
            c.close()


def test_barrier_wait_runs_out_when_a_peer_never_signals(cuda_device):
    """Rank 0 of a two-rank group runs alone: its barrier waits give up after
    about a second and the status word says so; the context stays usable."""
    lens = [40, 300]
    case = make_dcp_case(lens, 2, 1, 16, 8, seed=3)
    comms = dcp.DcpComm.emulated(2, 2, 8, 1, cuda_device)
    ws = comms[0].workspace(2, 8)
    try:
        out = torch.empty(2, 8, 128, dtype=torch.bfloat16, device=cuda_device)
        call = _rank_call(case, 0, cuda_device, out, None)
        t0 = time.monotonic()
        dcp.dcp_decode(comms[0], workspace=ws, **call)
        torch.cuda.synchronize()
        dt = time.monotonic() - t0
        assert ws.status() & _lib.PS_DEV_WAIT_TIMEOUT
        assert 0.9 < dt < 10.0
        x = torch.ones(4, device=cuda_device)
        assert float((x * 2).sum()) == 8.0
    finally:
        for c in comms:
            c.close()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _two_gpu_worker(rank, world, port, result_q):
    import sys
    from pathlib import Path

    repo = Path(__file__).resolve().parent.parent
    for p in (repo / "prime-rl_b200", repo, repo / "tests"):
        sys.path.insert(0, str(p))
    import torch.distributed as dist
    from dcp_helpers import make_dcp_case
    from ps_attn import dcp

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    comm = None
    try:
        lens = [1, 9, 100, 2049, 7000, 16]
        T = len(lens)
        comm = dcp.DcpComm.from_process_group(T, 32 // world, 1, device=dev)
        ws = comm.workspace(T, 8)
        for step in range(3):
            case = make_dcp_case(lens, world, 1, 32, 8, seed=200 + step)
            out = torch.empty(T, case.hq_local, 128, dtype=torch.bfloat16, device=dev)
            lse = torch.empty(case.hq_local, T, dtype=torch.float32, device=dev)
            call = _rank_call(case, rank, dev, out, lse)
            dcp.dcp_decode(comm, workspace=ws, **call)
            torch.cuda.synchronize(dev)
            assert ws.status() == 0, f"status {ws.status()}"
            want, want_lse = case.expected()
            kcs, vcs = case.expected_caches()
            _check_rank(case, rank, call, want, want_lse, kcs, vcs)
            dist.barrier()
        result_q.put((rank, "ok"))
    except Exception as e:  # surface the failure to the parent at once
        result_q.put((rank, repr(e)))
        raise
    finally:
        if comm is not None:
            dist.barrier()  # no peer still reads this rank's slab
            comm.close()
        dist.destroy_process_group()


def test_two_gpu_group_over_nvlink():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_two_gpu_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
    assert results == {0: "ok", 1: "ok"}
    assert all(p.exitcode == 0 for p in procs)


@pytest.mark.parametrize("world,interleave,hq,hkv", [(2, 1, 32, 8), (4, 16, 16, 8), (2, 1, 16, 2)])
def test_emulated_group_prefill_chunks(cuda_device, world, interleave, hq, hkv):
    """dcp_prefill: multi-token chunks on contexts spread over the ranks
    (context part across the group, the chunk's own causal part locally,
    merged) equal causal attention over the whole sequence; the chunk tokens
    each rank stores are appended bit-exactly."""
    from dcp_helpers import make_dcp_prefill_case

    c = make_dcp_prefill_case([0, 7, 300, 1500, 33], [5, 1, 40, 17, 9], world, interleave, hq, hkv, seed=11)
    T = c["q"].shape[0]
    hl = hq // world
    comms = dcp.DcpComm.emulated(world, T, hl, interleave, cuda_device)
    wss = [cm.workspace(T, hkv) for cm in comms]
    try:
        calls = []
        for r in range(world):
            calls.append(dict(
                q=c["q"][:, r * hl:(r + 1) * hl].to(cuda_device),
                key_cache=c["key_caches"][r].to(cuda_device), value_cache=c["value_caches"][r].to(cuda_device),
                block_table=c["block_table"].to(cuda_device), seq_lens=c["seq_lens"].to(cuda_device),
                query_start_loc=c["query_start_loc"].to(cuda_device), max_query_len=c["max_query_len"],
                softmax_scale=c["scale"],
                out=torch.full((T, hl, 128), float("nan"), dtype=torch.bfloat16, device=cuda_device),
                new_key=c["new_key"].to(cuda_device), new_value=c["new_value"].to(cuda_device),
                slot_mapping=c["slots"][r].to(cuda_device)))
        dcp.dcp_prefill_group(comms, calls, wss)
        torch.cuda.synchronize()
        for r in range(world):
            assert wss[r].status() == 0
            assert_attn_close(calls[r]["out"].float().cpu().numpy(), c["want"][:, r * hl:(r + 1) * hl])
            assert np.array_equal(calls[r]["key_cache"].float().cpu().numpy(), c["kc_ref"][r])
            assert np.array_equal(calls[r]["value_cache"].float().cpu().numpy(), c["vc_ref"][r])
    finally:
        for cm in comms:
            cm.close()


def test_merge_attn_states_matches_oracle(cuda_device):
    """ps_merge_attn_states against the oracle's merge (vLLM's rule; +inf
    and -inf LSEs included), in place on the prefix output."""
    from oracle import ps_oracle

    g = torch.Generator().manual_seed(4)
    T, H = 37, 8
    po = torch.randn(T, H, 128, generator=g).to(torch.bfloat16)
    so = torch.randn(T, H, 128, generator=g).to(torch.bfloat16)
    pl = torch.randn(H, T, generator=g) * 4
    sl = torch.randn(H, T, generator=g) * 4
    pl[0, :3] = -float("inf")
    pl[1, 3] = float("inf")
    want, want_lse = ps_oracle.merge_states(po.float().numpy(), pl.numpy(), so.float().numpy(), sl.numpy())
    out = po.to(cuda_device)
    lse = torch.empty(H, T, device=cuda_device)
    from ps_attn import ops

    ops.merge_attn_states(out, out, pl.to(cuda_device), so.to(cuda_device), sl.to(cuda_device), output_lse=lse)
    torch.cuda.synchronize()
    np.testing.assert_allclose(out.float().cpu().numpy(), want, atol=2e-2)
    assert np.abs(out.float().cpu().numpy() - want).mean() < 2e-3
    np.testing.assert_allclose(lse.cpu().numpy(), want_lse, atol=1e-5)
