"""Benchmark: paged PS-attention decode step (KV append + split-KV decode with
the fused combine) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config 2|3|5] [--impl ours|reference]

One "step" = append one new token per sequence through slot_mapping, then
decode attention for every sequence, on one layer (benchmark config 2 by
default: Qwen3-0.6B attention shapes 16q/8kv, d=128, bf16, 64 sequences,
contexts U[1024, 4096], block 16).  Inputs (KV pool 671 MB) exceed the 126 MB
L2, so no flush is needed between steps.

N > 1 (torchrun, one process per GPU): config 2 runs as independent replicas
of the batch per GPU (sequence-batch sharding, no data-path collective, weak
scaling); ``--config 5`` shards KV heads across GPUs and all-gathers the head
outputs with NCCL (strong scaling).

``--impl reference`` times the reference's CPU implementation of the same step
on the host cores (vLLM's fp32 torch ``attention_ref``, loaded by file path,
over the gathered pages, after a torch index-put append) on rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
for _p in (REPO / "prime-rl_b200", REPO):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

import torch  # noqa: E402

METRIC = "paged PS-attn decode tokens/s + HBM GB/s (% of 8 TB/s) at 1/2/4/8 B200"
NOMINAL_HBM_GBS = 8000.0
FALLBACK_HBM_GBS = 6650.0

CONFIG_NAMES = {
    2: "cfg2: Qwen3-0.6B attn (16q/8kv, d128) bf16 paged decode, B=64, ctx U[1024,4096], block 16",
    3: "cfg3: Qwen3-4B attn (32q/8kv, d128) bf16 GRPO decode, 32x8 seqs, shared 1024-token prefix, gen U[0,8192]",
    4: "cfg4: Qwen3-4B attn (32q/8kv, d128) bf16 mixed batch: 8 chunked-prefill x 2048 on ctx U[0,4096] + 128 decodes ctx U[512,8192]",
    5: "cfg5: Qwen3-32B attn (64q/8kv, d128) bf16 long-context decode, B=512, ctx log-U[2048,32768], KV-head sharded",
}


def prefill_flops(q_lens, seq_lens, num_q_heads, head_size=128):
    """4 * Hq * D * (unmasked causal (q, k) pairs) over the q_len > 1 sequences."""
    pairs = 0
    for n, L in zip(q_lens, seq_lens):
        if n > 1:
            c = L - n
            pairs += n * c + n * (n + 1) // 2
    return 4 * num_q_heads * head_size * pairs


def measured_peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def measured_tensor_peak():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text())["bf16_tflops"])
    return 1590.0


def profile_traffic(kernel_tag: str):
    """DRAM bytes per launch recorded by a committed ncu summary, or None."""
    f = REPO / "profiles" / f"{kernel_tag}.md"
    if not f.exists():
        return None
    for line in f.read_text().splitlines():
        if line.strip().startswith("traffic_bytes_per_launch:"):
            try:
                return int(float(line.split(":", 1)[1].strip().split()[0]))
            except ValueError:
                return None
    return None


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu_index = gpu_index
        self.proc = None
        self.path = Path(os.environ.get("TMPDIR", "/tmp")) / f"ps_clocks_{os.getpid()}.csv"

    def start(self):
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu_index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.fh, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.fh.close()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.path.read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        try:
            self.path.unlink()
        except OSError:
            pass
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "samples": len(sm),
                "reasons": sorted(reasons)}


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


# ----------------------------------------------------------------------------
# our arm
# ----------------------------------------------------------------------------
def run_ours(args):
    from ps_attn import _lib, ops, workloads

    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
    _lib.load(build_if_stale=False)
    cfg = args.config
    sharded = cfg == 5 and world > 1
    if sharded:
        hkv_total = 8
        assert hkv_total % world == 0, "KV heads must divide across GPUs"
        per = hkv_total // world
        batch = workloads.make_config(cfg, device=dev, kv_heads_slice=(rank * per, (rank + 1) * per))
    else:
        batch = workloads.make_config(cfg, device=dev, seed=rank if cfg != 5 else 0)
    B = batch.num_seqs
    hq = batch.q.shape[1]
    hkv = batch.kv_cache.shape[3]
    # GRPO groups share prompt pages: the cascade decode reads each prefix once
    # per 16-column pass (opt-in: on B200 it is not faster than the plain
    # decode, whose repeated prefix reads mostly hit L2)
    cascade = cfg == 3 and args.cascade
    ws = ops.DecodeWorkspace(B, hq, hkv, 128, dev, cascade=cascade)
    plan = ops.CascadePlan(B, dev) if cascade else None
    out = torch.empty_like(batch.q)
    lse = torch.empty(hq, B, dtype=torch.float32, device=dev)
    kc, vc = batch.kv_cache[0], batch.kv_cache[1]
    skw = {}  # fp8 cache: dequantization scales
    if args.kv_fp8:
        # e4m3 codes of the synthetic N(0,1) cache at scale 1/64 (|x| < 7 fits
        # in 448), quantized a slab of blocks at a time
        scale = torch.tensor(1.0 / 64.0, dtype=torch.float32, device=dev)
        codes = torch.empty(batch.kv_cache.shape, dtype=torch.uint8, device=dev)
        step_nb = 4096
        for i in range(0, batch.kv_cache.shape[1], step_nb):
            codes[:, i:i + step_nb] = (batch.kv_cache[:, i:i + step_nb].float() / scale).to(
                torch.float8_e4m3fn).view(torch.uint8)
        batch.kv_cache = codes
        kc, vc = codes[0], codes[1]
        skw = dict(k_scale=scale, v_scale=scale)
        torch.cuda.empty_cache()
    mixed = cfg == 4
    nd = B
    gathered = None
    peer_gather = None
    if sharded:
        gathered = torch.empty(world, B, hq, 128, dtype=batch.q.dtype, device=dev)
        full_out = torch.empty(B, hq * world, 128, dtype=batch.q.dtype, device=dev)
        if args.gather == "peer":
            # head outputs exchanged over NVLink peer memory (ps_head_gather)
            from ps_attn import sharding

            shard = sharding.HeadShard(world, rank, hq * world, hkv * world)
            peer_gather = sharding.PeerHeadGather.from_process_group(shard, B, batch.q.dtype, device=dev)

    fused = not args.unfused

    def append():
        if not fused:
            ops.kv_append(batch.key, batch.value, kc, vc, batch.slot_mapping)
        elif mixed:  # prefill tokens still go through the append kernel
            ops.kv_append(batch.key[nd:], batch.value[nd:], kc, vc, batch.slot_mapping[nd:])
        if cascade:  # the per-step plan (a serving engine builds it once per step for all layers)
            ops.cascade_plan(batch.block_table, batch.seq_lens, hq, hkv, 16,
                             query_start_loc=batch.query_start_loc, plan=plan)

    if mixed:
        qlens = (batch.query_start_loc[1:] - batch.query_start_loc[:-1]).tolist()
        nd = sum(1 for x in qlens if x == 1)
        assert all(x == 1 for x in qlens[:nd]), "decode-first batch expected"
        pf_flops = prefill_flops(qlens, batch.seq_lens.tolist(), hq)

    fkw = dict(new_key=batch.key, new_value=batch.value, slot_mapping=batch.slot_mapping) if fused else {}

    def decode():
        if peer_gather is not None:  # this rank's heads into its slab
            peer_gather.decode(batch.q, kc, vc, batch.block_table, batch.seq_lens, batch.softmax_scale,
                               full_out, lse=lse, query_start_loc=batch.query_start_loc, workspace=ws,
                               **fkw, **skw)
            return
        if not mixed:
            ops.paged_decode(batch.q, kc, vc, batch.block_table, batch.seq_lens,
                             batch.softmax_scale, out, lse=lse,
                             query_start_loc=batch.query_start_loc, workspace=ws, cascade=plan,
                             **fkw, **skw)
            return
        ops.paged_decode(batch.q[:nd], kc, vc, batch.block_table[:nd], batch.seq_lens[:nd],
                         batch.softmax_scale, out[:nd], workspace=ws, **fkw)

    def prefill():
        ops.chunked_prefill(batch.q, kc, vc, batch.block_table[nd:], batch.seq_lens[nd:],
                            batch.query_start_loc[nd:], batch.softmax_scale, out, workspace=ws)

    def gather():
        if peer_gather is not None:
            peer_gather.gather(B, full_out)
            return
        import torch.distributed as dist

        dist.all_gather_into_tensor(gathered, out)
        full_out.view(B, world, hq, 128).copy_(gathered.permute(1, 0, 2, 3))

    stream = torch.cuda.Stream(dev)
    use_graph = not args.no_graph
    graphs = {}
    with torch.cuda.stream(stream):
        for _ in range(3):  # warm up before capture
            append()
            decode()
            if peer_gather is not None:
                gather()
        stream.synchronize()
        if mixed:
            prefill()
            stream.synchronize()
        if use_graph:
            fns = ([("append", append)] if (not fused or mixed or cascade) else []) + [("decode", decode)] + (
                [("prefill", prefill)] if mixed else []) + ([("gather", gather)] if peer_gather else [])
            for name, fn in fns:
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=stream):
                    fn()
                graphs[name] = g

    def step(ev=None):
        if ev is not None:
            ev[0].record(stream)
        if use_graph:
            if "append" in graphs:
                graphs["append"].replay()
        else:
            append()
        if ev is not None:
            ev[1].record(stream)
        if use_graph:
            graphs["decode"].replay()
        else:
            decode()
        if ev is not None:
            ev[2].record(stream)
        if mixed:
            if use_graph:
                graphs["prefill"].replay()
            else:
                prefill()
            if ev is not None:
                ev[3].record(stream)
        if sharded:
            if use_graph and "gather" in graphs:
                graphs["gather"].replay()
            else:
                gather()

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step()
    torch.cuda.synchronize(dev)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
    torch.cuda.synchronize(dev)

    sampler = ClockSampler(local)
    if not args.quick:
        sampler.start()
        time.sleep(0.25)
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(args.steps)]
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        t0.record(stream)
        for i in range(args.steps):
            step(evs[i])
        t1.record(stream)
    torch.cuda.synchronize(dev)
    elapsed_ms = t0.elapsed_time(t1)
    # keep the same load on the GPU for at least ~1.5 s so the clock sampler sees it
    extra_t = time.perf_counter()
    with torch.cuda.stream(stream):
        while not args.quick and time.perf_counter() - extra_t < max(0.0, 1.5 - elapsed_ms / 1e3):
            for _ in range(50):
                step()
            stream.synchronize()
    clocks = sampler.stop()
    if world > 1:
        import torch.distributed as dist

        t = torch.tensor([elapsed_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed_ms = float(t.item())
    append_ms = sum(e[0].elapsed_time(e[1]) for e in evs) / args.steps
    decode_ms = sum(e[1].elapsed_time(e[2]) for e in evs) / args.steps
    prefill_ms = sum(e[2].elapsed_time(e[3]) for e in evs) / args.steps if mixed else None
    assert ws.status() == 0, f"device status {ws.status():#x}"

    # ---- end to end through the public API: host inputs in, host output back ----
    def nccl_gather(local_out):
        import torch.distributed as dist

        dist.all_gather_into_tensor(gathered, local_out)
        full_out.view(B, world, hq, 128).copy_(gathered.permute(1, 0, 2, 3))

    e2e = None if args.quick else run_e2e(
        batch, ws, dev, args.steps, world, nd=nd if mixed else None,
        replicas=1 if sharded else world, fused=fused, cascade=cascade, scales=skw,
        full_out=full_out if sharded else None, peer=peer_gather,
        gather=nccl_gather if sharded and peer_gather is None else None)

    ms = elapsed_ms / args.steps
    tokens_per_step = batch.num_tokens  # every rank produces all tokens (its heads when sharded)
    value = (tokens_per_step * (world if not sharded else 1)) / (ms / 1e3)
    peak, peak_kind = measured_peaks()
    if mixed:
        dec_tokens = int(batch.seq_lens[:nd].sum())
        kv_bytes = dec_tokens * hkv * 128 * 2 * batch.kv_cache.element_size()
        qo_bytes = nd * hq * 128 * 2 * batch.q.element_size()
        meta_bytes = nd * batch.block_table.shape[1] * 4 + nd * 4 * 2
    else:
        kv_tokens = batch.unique_tokens if cfg == 3 else batch.logical_tokens
        kv_bytes = kv_tokens * hkv * 128 * 2 * batch.kv_cache.element_size()
        qo_bytes = B * hq * 128 * 2 * batch.q.element_size()
        meta_bytes = batch.block_table.numel() * 4 + B * 4 * 2
    # a fused append also reads the new K/V rows and writes them into the cache
    app_bytes = (nd * hkv * 128 * 2 * (batch.key.element_size() + batch.kv_cache.element_size())
                 if fused else 0)
    decode_bytes = kv_bytes + qo_bytes + meta_bytes + app_bytes
    step_bytes = workloads.hbm_bytes(batch)
    achieved = decode_bytes / (decode_ms / 1e3) / 1e9
    traffic = None if args.kv_fp8 else profile_traffic(f"paged_decode_cfg{cfg}")
    res = {
        "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 5),
        "higher_is_better": True, "scaling": "strong" if sharded else "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {
            "workload": CONFIG_NAMES[cfg], "num_seqs": B, "num_q_heads": hq * (world if sharded else 1),
            "num_kv_heads": hkv * (world if sharded else 1), "head_size": 128, "block_size": 16,
            "kv_tokens": batch.logical_tokens, "kv_pool_bytes": batch.kv_cache.numel() * batch.kv_cache.element_size(),
            "parallelism": (f"kv-head tp{world} + " + ("NVLink peer-memory head gather (ps_head_gather)"
                                                       if peer_gather else "NCCL all-gather") if sharded else
                            (f"batch replicas x{world}" if world > 1 else "single GPU")),
            "l2": "inputs larger than L2 (KV pool > 126 MB); no flush",
            "cuda_graph": use_graph,
            "kv_cache_dtype": "fp8_e4m3 (per-tensor scale)" if args.kv_fp8 else "bf16",
        },
        "hbm_gbs_step": round(step_bytes / (ms / 1e3) / 1e9, 1),
        "hbm_frac_of_8tbs_step": round(step_bytes / (ms / 1e3) / 1e9 / NOMINAL_HBM_GBS, 4),
        "gpu_launches": ((3 if mixed else 2) - (1 if fused and not mixed else 0)
                         + (1 if cascade else 0) + (1 if peer_gather else 0)) * args.steps,
        "append_fused_into_decode": fused,
        "cascade": (None if not cascade else {
            "groups": int(plan.views()["num_groups"].item()),
            "note": "shared prompt pages read once per 16-column pass; plan built every step "
                    "(timed in append_ms); roofline bytes count each shared page once"}),
        "roofline": {"kernel": "paged_decode", "bound": "hbm", "achieved": round(achieved, 1),
                     "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                     "frac": round(achieved / peak, 4),
                     "frac_of_8tbs": round(achieved / NOMINAL_HBM_GBS, 4),
                     "bytes_per_launch": decode_bytes, "ms_per_launch": round(decode_ms, 5),
                     "traffic": traffic},
        "append_ms": round(append_ms, 5),
        "prefill": (None if not mixed else {
            "kernel": "chunked_prefill", "bound": "tensor", "ms_per_launch": round(prefill_ms, 5),
            "flops_per_launch": pf_flops,
            "achieved_tflops": round(pf_flops / (prefill_ms / 1e3) / 1e12, 1),
            "peak_tflops": measured_tensor_peak(), "peak_kind": "measured bf16 dense (cuBLAS)",
            "frac": round(pf_flops / (prefill_ms / 1e3) / 1e12 / measured_tensor_peak(), 4)}),
        "e2e": e2e,
        "clocks": clocks,
    }
    if rank == 0 and world == 1 and not args.quick:
        res["cpu_baseline"] = cpu_baseline(cfg, budget_s=args.cpu_budget)
    if rank == 0:
        print(json.dumps(res), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        graphs.clear()
        if peer_gather is not None:
            peer_gather.close()  # after the barrier: no peer still reads this slab
        dist.destroy_process_group()


def run_dcp(args):
    """Config 5 under decode context parallelism: every GPU holds all KV heads
    of a 1/N slice of every sequence; one ps_dcp_decode per step per rank
    (query gather, local decode, cross-rank combine + new-token merge +
    append, exchanged over NVLink peer memory, no NCCL)."""
    from ps_attn import _lib, dcp, workloads

    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    import datetime

    import torch.distributed as dist

    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    _lib.load(build_if_stale=False)
    cfg = args.config
    batch = workloads.make_dcp_config(cfg, world, rank, args.interleave, device=dev)
    B, hl = batch.q.shape[0], batch.q.shape[1]
    hkv = batch.kv_cache.shape[3]
    kc, vc = batch.kv_cache[0], batch.kv_cache[1]
    if world > 1:
        comm = dcp.DcpComm.from_process_group(B, hl, args.interleave, device=dev)
    else:
        comm = dcp.DcpComm.emulated(1, B, hl, args.interleave, dev)[0]
    ws = comm.workspace(B, hkv)
    out = torch.empty_like(batch.q)
    lse = torch.empty(hl, B, dtype=torch.float32, device=dev)
    kw = dict(q=batch.q, key_cache=kc, value_cache=vc, block_table=batch.block_table,
              seq_lens=batch.seq_lens, softmax_scale=batch.softmax_scale, out=out,
              new_key=batch.key, new_value=batch.value, slot_mapping=batch.slot_mapping,
              workspace=ws, lse=lse)
    stream = torch.cuda.Stream(dev)
    with torch.cuda.stream(stream):
        for _ in range(3):
            dcp.dcp_decode(comm, **kw)
        stream.synchronize()
        graph = None
        if not args.no_graph:
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                dcp.dcp_decode(comm, **kw)

    def step():
        if graph is not None:
            graph.replay()
        else:
            dcp.dcp_decode(comm, **kw)

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step()
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.25)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        t0.record(stream)
        for _ in range(args.steps):
            step()
        t1.record(stream)
    torch.cuda.synchronize(dev)
    elapsed_ms = t0.elapsed_time(t1)
    extra_t = time.perf_counter()
    with torch.cuda.stream(stream):
        while time.perf_counter() - extra_t < max(0.0, 1.5 - elapsed_ms / 1e3):
            for _ in range(20):
                step()
            stream.synchronize()
    clocks = sampler.stop()
    if world > 1:
        t = torch.tensor([elapsed_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed_ms = float(t.item())
    assert ws.status() == 0, f"device status {ws.status():#x}"

    # end to end: this step's new-token rows (q, k, v) and slots from pinned
    # host memory in, the output back to the host, every step
    hq_in = batch.q.cpu().pin_memory()
    hk_in, hv_in = batch.key.cpu().pin_memory(), batch.value.cpu().pin_memory()
    hs_in = batch.slot_mapping.cpu().pin_memory()
    h_out = torch.empty(out.shape, dtype=out.dtype).pin_memory()
    dq, dk, dv, ds = (torch.empty_like(batch.q), torch.empty_like(batch.key),
                      torch.empty_like(batch.value), torch.empty_like(batch.slot_mapping))
    ekw = dict(kw, q=dq, new_key=dk, new_value=dv, slot_mapping=ds)
    with torch.cuda.stream(stream):
        def one():
            dq.copy_(hq_in, non_blocking=True)
            dk.copy_(hk_in, non_blocking=True)
            dv.copy_(hv_in, non_blocking=True)
            ds.copy_(hs_in, non_blocking=True)
            dcp.dcp_decode(comm, **ekw)
            h_out.copy_(out, non_blocking=True)

        for _ in range(3):
            one()
        stream.synchronize()
        if world > 1:
            dist.barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            one()
        e1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    h2d = sum(x.numel() * x.element_size() for x in (hq_in, hk_in, hv_in, hs_in))
    d2h = h_out.numel() * h_out.element_size()

    ms = elapsed_ms / args.steps
    es = batch.kv_cache.element_size()
    hq_all = hl * world
    # per rank: its context slice of K and V, the group's query rows gathered
    # and their partial outputs written, the peers' partials read for its heads
    kv_bytes = batch.unique_tokens * hkv * 128 * 2 * es
    ex_bytes = B * hq_all * 128 * es * 3 + B * hl * 128 * es * (world + 2)
    step_bytes = kv_bytes + ex_bytes + batch.block_table.numel() * 4 + B * 4 * 2
    achieved = step_bytes / (ms / 1e3) / 1e9
    peak, peak_kind = measured_peaks()
    res = {
        "metric": METRIC, "value": round(B / (ms / 1e3), 1), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 5),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic",
        "config": {"workload": CONFIG_NAMES[cfg] + " -- decode context parallel", "num_seqs": B,
                   "num_q_heads": hq_all, "num_kv_heads": hkv, "head_size": 128, "block_size": 16,
                   "kv_tokens": batch.logical_tokens, "kv_tokens_this_rank": batch.unique_tokens,
                   "parallelism": f"dcp{world} (interleave {args.interleave}), peer-memory exchange",
                   "l2": "inputs larger than L2 (KV pool > 126 MB); no flush",
                   "cuda_graph": graph is not None},
        "gpu_launches": 4 * args.steps,
        "roofline": {"kernel": "dcp step (gather + paged_decode + combine)", "bound": "hbm",
                     "achieved": round(achieved, 1), "peak": peak, "peak_kind": peak_kind,
                     "unit": "GB/s", "frac": round(achieved / peak, 4),
                     "frac_of_8tbs": round(achieved / NOMINAL_HBM_GBS, 4),
                     "bytes_per_launch": step_bytes, "ms_per_launch": round(ms, 5), "traffic": None},
        "e2e": {"value": round(B / (e2e_ms / args.steps / 1e3), 1), "unit": "tokens/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "clocks": clocks,
    }
    if rank == 0:
        print(json.dumps(res), flush=True)
    graph = None
    if world > 1:
        dist.barrier()
    comm.close()
    if world > 1:
        dist.destroy_process_group()


def run_e2e(batch, ws, dev, steps, world, nd=None, replicas=1, fused=True, cascade=False, scales=None,
            full_out=None, peer=None, gather=None):
    """Same step through the public ops with per-step host->device inputs
    (pinned) and the device->host read of the attention output.  ``nd``:
    number of leading decode sequences of a mixed batch (the rest prefill).
    KV-head sharded runs (``full_out``) include the head all-gather -- over
    peer memory (``peer``) or NCCL (``gather(local_out)``) -- and read back
    the whole output."""
    from ps_attn import ops

    B, hq = batch.num_seqs, batch.q.shape[1]
    T = batch.num_tokens
    host = {k: getattr(batch, k).cpu().pin_memory() for k in
            ("q", "key", "value", "slot_mapping", "seq_lens", "block_table", "query_start_loc")}
    dev_in = {k: torch.empty_like(v, device=dev) for k, v in host.items()}
    out = torch.empty_like(batch.q)
    result = out if full_out is None else full_out
    out_host = torch.empty(result.shape, dtype=result.dtype).pin_memory()
    h2d = sum(v.numel() * v.element_size() for v in host.values())
    d2h = result.numel() * result.element_size()
    kc, vc = batch.kv_cache[0], batch.kv_cache[1]
    plan = ops.CascadePlan(B, dev) if cascade else None

    def one():
        for k, v in host.items():
            dev_in[k].copy_(v, non_blocking=True)
        fkw = dict(new_key=dev_in["key"], new_value=dev_in["value"],
                   slot_mapping=dev_in["slot_mapping"]) if fused else {}
        if not fused:
            ops.kv_append(dev_in["key"], dev_in["value"], kc, vc, dev_in["slot_mapping"])
        elif nd is not None:
            ops.kv_append(dev_in["key"][nd:], dev_in["value"][nd:], kc, vc, dev_in["slot_mapping"][nd:])
        if peer is not None:
            peer.decode(dev_in["q"], kc, vc, dev_in["block_table"], dev_in["seq_lens"],
                        batch.softmax_scale, full_out, query_start_loc=dev_in["query_start_loc"],
                        workspace=ws, **fkw, **(scales or {}))
            peer.gather(T, full_out)
        elif nd is None:
            if cascade:
                ops.cascade_plan(dev_in["block_table"], dev_in["seq_lens"], hq,
                                 kc.shape[2], kc.shape[1], query_start_loc=dev_in["query_start_loc"],
                                 plan=plan)
            ops.paged_decode(dev_in["q"], kc, vc, dev_in["block_table"], dev_in["seq_lens"],
                             batch.softmax_scale, out, query_start_loc=dev_in["query_start_loc"],
                             workspace=ws, cascade=plan, **fkw, **(scales or {}))
        else:
            ops.paged_decode(dev_in["q"][:nd], kc, vc, dev_in["block_table"][:nd],
                             dev_in["seq_lens"][:nd], batch.softmax_scale, out[:nd], workspace=ws,
                             **fkw)
            ops.chunked_prefill(dev_in["q"], kc, vc, dev_in["block_table"][nd:],
                                dev_in["seq_lens"][nd:], dev_in["query_start_loc"][nd:],
                                batch.softmax_scale, out, workspace=ws)
        if gather is not None:
            gather(out)
        out_host.copy_(result, non_blocking=True)

    n = max(3, min(steps, 200))
    for _ in range(3):
        one()
    torch.cuda.synchronize(dev)
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(n):
        one()
    b.record()
    torch.cuda.synchronize(dev)
    ms = a.elapsed_time(b) / n
    if world > 1:
        import torch.distributed as dist

        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return {"value": round(T * replicas / (ms / 1e3), 1), "unit": "tokens/s",
            "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
            "ms_per_step": round(ms, 5), "steps": n}


# ----------------------------------------------------------------------------
# reference (CPU) arm
# ----------------------------------------------------------------------------
def load_reference_attention():
    """vLLM's FA4 torch reference attention_ref, loaded by file path; None if absent."""
    import importlib.util

    spec = importlib.util.find_spec("vllm")
    if spec is None or spec.origin is None:
        return None
    path = Path(spec.origin).parent / "vllm_flash_attn" / "cute" / "testing.py"
    if not path.exists():
        return None
    s = importlib.util.spec_from_file_location("fa4_testing_ref", path)
    mod = importlib.util.module_from_spec(s)
    s.loader.exec_module(mod)
    return mod.attention_ref


def reference_step(batch, attention_ref, seqs):
    """Reference CPU step for sequences ``seqs``: index-put append (the
    reshape_and_cache_flash contract), page gather, fp32 attention_ref."""
    kc, vc = batch.kv_cache[0], batch.kv_cache[1]
    hkv, d = kc.shape[2], kc.shape[3]
    bs = kc.shape[1]
    sl = batch.slot_mapping
    ok = sl >= 0
    kc.view(-1, hkv, d)[sl[ok]] = batch.key[ok]
    vc.view(-1, hkv, d)[sl[ok]] = batch.value[ok]
    outs = []
    for b in seqs:
        L = int(batch.seq_lens[b])
        npg = (L + bs - 1) // bs
        blocks = batch.block_table[b, :npg].long()
        k = kc[blocks].reshape(npg * bs, hkv, d)[:L].float()
        v = vc[blocks].reshape(npg * bs, hkv, d)[:L].float()
        q = batch.q[b:b + 1].float()
        o, _, lse = attention_ref(q[None], k[None], v[None], causal=True, return_lse=True)
        outs.append(o)
    return outs


def cpu_baseline(cfg, budget_s=20.0, steps=None, warmup=1):
    """Time the reference CPU step on a bounded sample of the workload."""
    from ps_attn import workloads

    attention_ref = load_reference_attention()
    kind = "reference"
    if attention_ref is None:  # vLLM missing: the oracle port stands in
        from oracle import ps_oracle

        kind = "port"

        def attention_ref(q, k, v, causal=True, return_lse=True):
            o, l = ps_oracle.attention_ref(q[0].numpy(), k[0].numpy(), v[0].numpy(), causal=causal)
            return torch.from_numpy(o)[None], None, torch.from_numpy(l)[None]

    # sequences: seeded prefix subset sized for the time budget
    sub = {2: 64, 3: 16, 4: 16, 5: 16}[cfg]
    batch = workloads.make_config(cfg, device="cpu", max_seqs=sub)
    seqs = list(range(batch.num_seqs))
    for _ in range(warmup):
        reference_step(batch, attention_ref, seqs[:2])
    n_done, t_used = 0, 0.0
    step_times = []
    while t_used < budget_s and (steps is None or len(step_times) < steps):
        t = time.perf_counter()
        reference_step(batch, attention_ref, seqs)
        dt = time.perf_counter() - t
        step_times.append(dt)
        t_used += dt
        n_done += len(seqs)
        if steps is None and len(step_times) >= 200:
            break
    value = n_done / t_used
    return {"value": round(value, 2), "unit": "tokens/s", "cores": torch.get_num_threads(),
            "kind": kind,
            "sample": f"cfg{cfg}: {len(seqs)} sequences x {len(step_times)} steps "
                      f"({t_used:.1f} s), fp32 attention_ref per sequence on gathered pages, "
                      f"torch index-put append; KV pool kept in the config dtype",
            "ms_per_step": round(1e3 * t_used / len(step_times), 3)}


def run_reference(args):
    world, rank, _ = dist_env()
    if rank != 0:
        return
    torch.set_num_threads(os.cpu_count() or 1)
    cb = cpu_baseline(args.config, budget_s=args.cpu_budget, steps=args.steps, warmup=max(1, min(args.warmup, 3)))
    res = {
        "metric": METRIC, "impl": "reference", "value": cb["value"], "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": cb["ms_per_step"], "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
        "config": {"workload": CONFIG_NAMES[args.config] + " (CPU reference, seeded sequence subset)"},
        "cpu_baseline": cb,
        "e2e": {"value": cb["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(res), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--config", type=int, default=2, choices=[2, 3, 4, 5])
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--unfused", action="store_true",
                    help="separate append launch instead of the append fused into decode")
    ap.add_argument("--cascade", action="store_true",
                    help="config 3: shared-prefix (cascade) decode with a per-step plan")
    ap.add_argument("--dcp", action="store_true",
                    help="config 5 under decode context parallelism (tokens sharded, not heads)")
    ap.add_argument("--gather", default="peer", choices=["nccl", "peer"],
                    help="config 5 on N GPUs: head outputs all-gathered by NCCL or over peer memory")
    ap.add_argument("--kv-fp8", action="store_true",
                    help="decode configs over an fp8 (e4m3) KV cache, fused quantizing append")
    ap.add_argument("--interleave", type=int, default=1,
                    help="DCP: consecutive positions per rank (vLLM cp_kv_cache_interleave_size)")
    ap.add_argument("--cpu-budget", type=float, default=15.0)
    ap.add_argument("--quick", action="store_true",
                    help="timed steps only: no end-to-end, CPU baseline or clock sampling")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    elif args.dcp:
        if args.config not in (2, 3, 5) or args.kv_fp8:
            ap.error("--dcp takes a decode config (2, 3 or 5) with a 16-bit cache")
        run_dcp(args)
    else:
        if args.kv_fp8 and (args.config == 4 or args.cascade or args.unfused):
            ap.error("--kv-fp8: plain decode configs (2, 3, 5) with the fused append")
        run_ours(args)


if __name__ == "__main__":
    main()
