"""Benchmark: paged PS-attention decode step (KV append + split-KV decode with
the fused combine) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config 2|3|4|5] [--impl ours|reference]

One "step" = append one new token per sequence through slot_mapping, then
decode attention for every sequence, on one layer.  The default workload is
benchmark config 5 (Qwen3-32B attention shapes 64q/8kv, d=128, bf16, 512
sequences, contexts log-uniform in [2048, 32768], block 16): the config the
metric is quoted on at 1/2/4/8 GPUs.  Inputs (KV pool 23 GB) exceed the
126 MB L2, so no flush is needed between steps.

N > 1 (torchrun, one process per GPU): config 5 shards KV heads across the
GPUs (rank r: KV heads [r*8/N, (r+1)*8/N) and their query heads) and
all-gathers the head outputs over NVLink peer memory inside the decode launch
(``ps_paged_decode_head_gather``: rows stored into the peers as they are
finished; ``--gather peer`` for the separate pull launch ``ps_head_gather``,
``--gather nccl`` for NCCL's all_gather) -- strong scaling, every rank checks
sampled gathered rows against a torch fp32 attention of the same rows.
Configs 2-4 at N > 1 run as independent replicas (sequence-batch sharding,
no data-path collective, weak scaling).

At N = 1 the line also carries (unless ``--no-side`` / ``--no-fa4``):
``fa4`` -- vLLM's own path on the same inputs and GPU
(``reshape_and_cache_flash`` + ``flash_attn_varlen_func(fa_version=4)``),
timed with CUDA events; ``configs`` -- configs 2, 3 and 4 measured the same
way; ``prefill`` -- config 4's chunked prefill on the tensor-core roofline.

``--impl reference`` times the reference's CPU implementation of the same step
on the host cores (vLLM's fp32 torch ``attention_ref``, loaded by file path,
over the gathered pages, after a torch index-put append) on rank 0 only.
"""
from __future__ import annotations

import argparse
import json
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
DEFAULT_CONFIG = 5
FA4_CALL = ("vllm._custom_ops.reshape_and_cache_flash + vllm.vllm_flash_attn.flash_attn_varlen_func("
            "q, k_cache, v_cache, out, cu_seqlens_q, max_seqlen_q, seqused_k, max_seqlen_k, "
            "softmax_scale, causal=True, block_table, fa_version=4, num_splits=0) as "
            "vllm/v1/attention/backends/flash_attn.py:796-817 calls it on sm_100")

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


def _peaks_file():
    p = REPO / "MEASURED_PEAKS.json"
    return json.loads(p.read_text()) if p.exists() else None


def measured_peaks():
    d = _peaks_file()
    if d is not None:
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def measured_tensor_peaks():
    """(burst, sustained) dense bf16 TFLOP/s and their source."""
    d = _peaks_file()
    if d is not None:
        return float(d["bf16_tflops"]), float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "measured"
    return 1590.0, 1400.0, "fallback"


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


def config_dict(cfg: int, max_seqs: int | None = None) -> dict:
    """The workload description shared by both arms (no device needed)."""
    from ps_attn import workloads

    q_lens, seq_lens, kw = workloads.config_lengths(cfg)
    name = CONFIG_NAMES[cfg]
    if max_seqs is not None:  # a profiling subset, not a benchmark line
        q_lens, seq_lens = q_lens[:max_seqs], seq_lens[:max_seqs]
        name += f" -- first {len(seq_lens)} sequences only"
    return {"workload": name, "num_seqs": len(seq_lens), "num_q_heads": kw["num_q_heads"],
            "num_kv_heads": kw["num_kv_heads"], "head_size": 128, "block_size": 16,
            "kv_tokens": int(sum(seq_lens)), "new_tokens_per_step": int(sum(q_lens))}


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


def _all_max(x: float, world: int, dev) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


INPUT_KEYS = ("q", "key", "value", "slot_mapping", "seq_lens", "block_table", "query_start_loc")


# ----------------------------------------------------------------------------
# our arm
# ----------------------------------------------------------------------------
class Arm:
    """One benchmark config on this GPU: its batch, buffers and the step's
    launches as a list of phases (append / plan / decode / prefill / gather),
    each replayed from its own CUDA graph so CUDA events can bracket it."""

    def __init__(self, cfg, dev, world=1, rank=0, *, kv_fp8=False, cascade=False, fused=True,
                 gather="fused", use_graph=True, max_seqs=None):
        from ps_attn import ops, workloads

        self.cfg, self.dev, self.world, self.rank = cfg, dev, world, rank
        self.sharded = cfg == 5 and world > 1
        self.gather_kind = gather
        self.kv_fp8, self.fused, self.use_graph = kv_fp8, fused, use_graph
        if self.sharded:
            per = 8 // world
            batch = workloads.make_config(cfg, device=dev, kv_heads_slice=(rank * per, (rank + 1) * per),
                                          max_seqs=max_seqs)
        else:
            batch = workloads.make_config(cfg, device=dev, seed=rank if cfg != 5 else 0, max_seqs=max_seqs)
        self.batch = batch
        B = self.B = batch.num_seqs
        self.hq, self.hkv = batch.q.shape[1], batch.kv_cache.shape[3]
        # GRPO groups share prompt pages: the cascade decode reads each prefix
        # once per 16-column pass (opt-in: on B200 it is not faster than the
        # plain decode, whose repeated prefix reads mostly hit L2)
        self.cascade = cfg == 3 and cascade
        self.ws = ops.DecodeWorkspace(B, self.hq, self.hkv, 128, dev, cascade=self.cascade)
        self.plan = ops.CascadePlan(B, dev) if self.cascade else None
        self.out = torch.empty_like(batch.q)
        self.lse = torch.empty(self.hq, batch.num_tokens, dtype=torch.float32, device=dev)
        self.skw = {}
        if kv_fp8:
            # e4m3 codes of the synthetic N(0,1) cache at scale 1/64 (|x| < 7
            # fits in 448), quantized a slab of blocks at a time
            scale = torch.tensor(1.0 / 64.0, dtype=torch.float32, device=dev)
            codes = torch.empty(batch.kv_cache.shape, dtype=torch.uint8, device=dev)
            for i in range(0, batch.kv_cache.shape[1], 4096):
                codes[:, i:i + 4096] = (batch.kv_cache[:, i:i + 4096].float() / scale).to(
                    torch.float8_e4m3fn).view(torch.uint8)
            batch.kv_cache = codes
            self.skw = dict(k_scale=scale, v_scale=scale)
            torch.cuda.empty_cache()
        self.kc, self.vc = batch.kv_cache[0], batch.kv_cache[1]
        self.mixed = cfg == 4
        self.nd = B
        self.pf_flops = 0
        if self.mixed:
            qlens = (batch.query_start_loc[1:] - batch.query_start_loc[:-1]).tolist()
            self.nd = sum(1 for x in qlens if x == 1)
            assert all(x == 1 for x in qlens[:self.nd]), "decode-first batch expected"
            self.pf_flops = prefill_flops(qlens, batch.seq_lens.tolist(), self.hq)
        self.peer_gather = None
        self.full_out = None
        self.gathered = None
        if self.sharded:
            self.full_out = torch.empty(B, self.hq * world, 128, dtype=batch.q.dtype, device=dev)
            if gather in ("fused", "peer"):
                # head outputs exchanged over NVLink peer memory: stored into
                # the peers by the decode itself (ps_paged_decode_head_gather),
                # or pulled by a separate launch (ps_head_gather)
                from ps_attn import sharding

                shard = sharding.HeadShard(world, rank, self.hq * world, self.hkv * world)
                cls = sharding.FusedHeadGather if gather == "fused" else sharding.PeerHeadGather
                self.peer_gather = cls.from_process_group(shard, B, batch.q.dtype, device=dev)
            else:
                self.gathered = torch.empty(world, B, self.hq, 128, dtype=batch.q.dtype, device=dev)
        self.stream = torch.cuda.Stream(dev)
        self.graphs = []
        self.names = []

    # -- the step's launches over a set of input tensors -----------------------
    def inputs(self) -> dict:
        return {k: getattr(self.batch, k) for k in INPUT_KEYS}

    def phases(self, inp: dict) -> list:
        from ps_attn import ops

        kc, vc, ws, plan, nd = self.kc, self.vc, self.ws, self.plan, self.nd
        scale = self.batch.softmax_scale
        out, lse, skw = self.out, self.lse, self.skw
        fkw = dict(new_key=inp["key"], new_value=inp["value"],
                   slot_mapping=inp["slot_mapping"]) if self.fused else {}
        ph = []
        if not self.fused:
            ph.append(("append", lambda: ops.kv_append(inp["key"], inp["value"], kc, vc, inp["slot_mapping"],
                                                       **skw)))
        elif self.mixed:  # prefill tokens still go through the append kernel
            ph.append(("append", lambda: ops.kv_append(inp["key"][nd:], inp["value"][nd:], kc, vc,
                                                       inp["slot_mapping"][nd:])))
        if self.cascade:  # the per-step plan (an engine builds it once per step for all layers)
            ph.append(("plan", lambda: ops.cascade_plan(inp["block_table"], inp["seq_lens"], self.hq, self.hkv,
                                                        16, query_start_loc=inp["query_start_loc"], plan=plan)))
        if self.peer_gather is not None:  # this rank's heads (fused: and the exchange)
            ph.append(("decode", lambda: self.peer_gather.decode(
                inp["q"], kc, vc, inp["block_table"], inp["seq_lens"], scale, self.full_out, lse=lse,
                query_start_loc=inp["query_start_loc"], workspace=ws, **fkw, **skw)))
        elif not self.mixed:
            ph.append(("decode", lambda: ops.paged_decode(
                inp["q"], kc, vc, inp["block_table"], inp["seq_lens"], scale, out, lse=lse,
                query_start_loc=inp["query_start_loc"], workspace=ws, cascade=plan, **fkw, **skw)))
        else:
            ph.append(("decode", lambda: ops.paged_decode(
                inp["q"][:nd], kc, vc, inp["block_table"][:nd], inp["seq_lens"][:nd], scale, out[:nd],
                lse=lse[:, :nd], workspace=ws, **fkw)))
            ph.append(("prefill", lambda: ops.chunked_prefill(
                inp["q"], kc, vc, inp["block_table"][nd:], inp["seq_lens"][nd:], inp["query_start_loc"][nd:],
                scale, out, lse=lse, workspace=ws)))
        if self.sharded:
            if self.gather_kind == "fused":
                pass  # inside the decode launch
            elif self.peer_gather is not None:
                ph.append(("gather", lambda: self.peer_gather.gather(self.B, self.full_out)))
            else:
                def nccl_gather():
                    import torch.distributed as dist

                    dist.all_gather_into_tensor(self.gathered, out)
                    self.full_out.view(self.B, self.world, self.hq, 128).copy_(self.gathered.permute(1, 0, 2, 3))

                ph.append(("gather", nccl_gather))
        return ph

    def result(self) -> torch.Tensor:
        """The step's output as the caller reads it."""
        return self.full_out if self.sharded else self.out

    def capture(self, inp: dict | None = None) -> tuple:
        """Warm up the phases over ``inp`` and capture one graph per phase.
        Returns (names, callables, graphs); with --no-graph the callables are
        the eager phases and there are no graphs."""
        ph = self.phases(self.inputs() if inp is None else inp)
        names = [n for n, _ in ph]
        if self.sharded:
            # the ranks reach their first exchange together (its waits are bounded)
            import torch.distributed as dist

            torch.cuda.synchronize(self.stream.device)
            dist.barrier()
        with torch.cuda.stream(self.stream):
            for _ in range(3):
                for _, fn in ph:
                    fn()
            self.stream.synchronize()
            if not self.use_graph:
                return names, [fn for _, fn in ph], []
            graphs = []
            for _, fn in ph:
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=self.stream):
                    fn()
                graphs.append(g)
        return names, [g.replay for g in graphs], graphs

    def setup(self):
        self.names, self.runs, self.graphs = self.capture()

    def step(self, ev=None):
        if ev is not None:
            ev[0].record(self.stream)
        for i, run in enumerate(self.runs):
            run()
            if ev is not None:
                ev[i + 1].record(self.stream)

    def time(self, steps: int, warmup: int, sampler: ClockSampler | None = None) -> dict:
        world, dev = self.world, self.dev
        with torch.cuda.stream(self.stream):
            for _ in range(warmup):
                self.step()
        torch.cuda.synchronize(dev)
        if world > 1:
            import torch.distributed as dist

            dist.barrier()
        torch.cuda.synchronize(dev)
        if sampler is not None:
            sampler.start()
            time.sleep(0.25)
        # the timed region: K steps back to back, events only at its ends
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(self.stream):
            t0.record(self.stream)
            for _ in range(steps):
                self.step()
            t1.record(self.stream)
        torch.cuda.synchronize(dev)
        elapsed_ms = t0.elapsed_time(t1)
        if len(self.runs) == 1:
            # one launch per step: its average duration is the step's
            phase_ms = {self.names[0]: elapsed_ms / steps}
        else:
            # several launches per step: a second pass of K steps with an
            # event between launches gives each launch's duration
            n_ev = len(self.runs) + 1
            evs = [[torch.cuda.Event(enable_timing=True) for _ in range(n_ev)] for _ in range(steps)]
            with torch.cuda.stream(self.stream):
                for i in range(steps):
                    self.step(evs[i])
            torch.cuda.synchronize(dev)
            phase_ms = {n: sum(e[i].elapsed_time(e[i + 1]) for e in evs) / steps for i, n in enumerate(self.names)}
        clocks = None
        if sampler is not None:
            # keep the same load on the GPU for ~1.5 s so the sampler sees it
            extra_t = time.perf_counter()
            with torch.cuda.stream(self.stream):
                while time.perf_counter() - extra_t < max(0.0, 1.5 - elapsed_ms / 1e3):
                    for _ in range(20):
                        self.step()
                    self.stream.synchronize()
            clocks = sampler.stop()
        elapsed_ms = _all_max(elapsed_ms, world, dev)
        assert self.ws.status() == 0, f"device status {self.ws.status():#x}"
        return {"elapsed_ms": elapsed_ms, "ms": elapsed_ms / steps, "phase_ms": phase_ms, "clocks": clocks}

    # -- roofline bookkeeping ---------------------------------------------------
    def decode_bytes(self) -> int:
        """Algorithmic bytes of one decode launch: KV read (config 3: each
        shared prefix page once), Q in, O out, block table + lengths, and the
        fused append's row read + write."""
        b, nd, hkv, hq = self.batch, self.nd, self.hkv, self.hq
        es = b.kv_cache.element_size()
        if self.mixed:
            kv_tokens = int(b.seq_lens[:nd].sum())
            meta = nd * b.block_table.shape[1] * 4 + nd * 4 * 2
        else:
            kv_tokens = b.unique_tokens if self.cfg == 3 else b.logical_tokens
            meta = b.block_table.numel() * 4 + nd * 4 * 2
        kv = kv_tokens * hkv * 128 * 2 * es
        qo = nd * hq * 128 * 2 * b.q.element_size()
        app = nd * hkv * 128 * 2 * (b.key.element_size() + es) if self.fused else 0
        return int(kv + qo + meta + app)

    def launches_per_step(self) -> int:
        return len(self.names)

    def close(self):
        self.graphs.clear()
        self.runs = []
        if self.peer_gather is not None:
            self.peer_gather.close()


def decode_roofline(arm: Arm, decode_ms: float, traffic=None) -> dict:
    peak, peak_kind = measured_peaks()
    nbytes = arm.decode_bytes()
    achieved = nbytes / (decode_ms / 1e3) / 1e9
    return {"kernel": "paged_decode", "bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
            "peak_kind": peak_kind, "unit": "GB/s", "frac": round(achieved / peak, 4),
            "frac_of_8tbs": round(achieved / NOMINAL_HBM_GBS, 4), "bytes_per_launch": nbytes,
            "ms_per_launch": round(decode_ms, 5), "traffic": traffic}


def prefill_roofline(arm: Arm, prefill_ms: float) -> dict:
    burst, sustained, kind = measured_tensor_peaks()
    tf = arm.pf_flops / (prefill_ms / 1e3) / 1e12
    return {"kernel": "chunked_prefill", "bound": "tensor", "ms_per_launch": round(prefill_ms, 5),
            "flops_per_launch": arm.pf_flops, "achieved": round(tf, 1), "unit": "TFLOP/s",
            "peak": sustained, "peak_kind": f"{kind} bf16 dense (cuBLAS), sustained",
            "frac": round(tf / sustained, 4), "frac_of_burst": round(tf / burst, 4),
            "traffic": profile_traffic("chunked_prefill_cfg4")}


# ----------------------------------------------------------------------------
# vLLM's FA4 path on the same inputs (the GPU bar)
# ----------------------------------------------------------------------------
def _median_ms(fn, stream, n: int) -> float:
    """Average duration of ``fn`` over n back-to-back calls (the way the
    timed region runs our steps), the median of three such runs."""
    runs = []
    with torch.cuda.stream(stream):
        for _ in range(3):
            fn()
        stream.synchronize()
        for _ in range(3):
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record(stream)
            for _ in range(n):
                fn()
            b.record(stream)
            stream.synchronize()
            runs.append(a.elapsed_time(b) / n)
    return statistics.median(runs)


def fa4_compare(arm: Arm, steps: int, ours_step_ms: float, ours_phase_ms: dict) -> dict:
    """Time vLLM's serving call on ``arm``'s inputs (the same cache, block
    table and new rows; the append writes the same bytes ours does) and
    compare its output and LSE with ours.  Timed as the faster of eager
    calls and a CUDA-graph replay (vLLM serves decode from full graphs)."""
    try:
        from vllm import _custom_ops as vops
        from vllm.vllm_flash_attn.flash_attn_interface import flash_attn_varlen_func
    except Exception as e:  # noqa: BLE001
        return {"unavailable": f"vLLM FA4 import failed: {e!r}"[:300]}
    b, dev, nd = arm.batch, arm.dev, arm.nd
    kc, vc = arm.kc, arm.vc
    ones = torch.ones(1, dtype=torch.float32, device=dev)
    qsl_h = b.query_start_loc.cpu()
    sl_h = b.seq_lens.cpu()
    out_fa = torch.empty_like(b.q)
    stream = arm.stream

    def call(rows, seqs, append=True, want_lse=False):
        q0, q1 = rows
        s0, s1 = seqs
        qsl = b.query_start_loc[s0:s1 + 1] - b.query_start_loc[s0] if s0 else b.query_start_loc[s0:s1 + 1]
        mq = int((qsl_h[s0 + 1:s1 + 1] - qsl_h[s0:s1]).max())
        mk = int(sl_h[s0:s1].max())

        def fn():
            if append:
                vops.reshape_and_cache_flash(b.key[q0:q1], b.value[q0:q1], kc, vc, b.slot_mapping[q0:q1],
                                             "auto", ones, ones)
            return flash_attn_varlen_func(
                q=b.q[q0:q1], k=kc, v=vc, out=out_fa[q0:q1], cu_seqlens_q=qsl, max_seqlen_q=mq,
                seqused_k=b.seq_lens[s0:s1], max_seqlen_k=mk, softmax_scale=b.softmax_scale, causal=True,
                block_table=b.block_table[s0:s1], softcap=0.0, fa_version=4, num_splits=0,
                return_softmax_lse=want_lse)
        return fn

    T, B = b.num_tokens, arm.B
    res = {"call": FA4_CALL}
    try:
        full = call((0, T), (0, B))
        t = time.perf_counter()
        with torch.cuda.stream(stream):
            _, lse_fa = call((0, T), (0, B), want_lse=True)()
        stream.synchronize()
        res["jit_s"] = round(time.perf_counter() - t, 1)
        d = (out_fa.float() - arm.out.float()).abs()
        res["max_abs_diff_vs_ours"] = float(d.max())
        res["mean_abs_diff_vs_ours"] = float(d.mean())
        res["lse_max_abs_diff_vs_ours"] = float((lse_fa - arm.lse).abs().max())
        eager = _median_ms(full, stream, steps)
        with torch.cuda.stream(stream):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                full()
        graphed = _median_ms(g.replay, stream, steps)
        del g
        ms = min(eager, graphed)
        res.update({"ms_per_step": round(ms, 5), "eager_ms": round(eager, 5), "graph_ms": round(graphed, 5),
                    "tokens_per_s": round(T / (ms / 1e3), 1),
                    "ratio_ours_over_fa4": round(ms / ours_step_ms, 4)})
        if arm.mixed:
            # the two halves separately (attention only), against our kernels
            dec = _median_ms(call((0, nd), (0, nd), append=False), stream, steps)
            pre = _median_ms(call((nd, T), (nd, B), append=False), stream, steps)
            res["decode_attention_ms"] = round(dec, 5)
            res["prefill_attention_ms"] = round(pre, 5)
            res["decode_ratio_ours_over_fa4"] = round(dec / ours_phase_ms["decode"], 4)
            res["prefill_ratio_ours_over_fa4"] = round(pre / ours_phase_ms["prefill"], 4)
        else:
            res["decode_attention_ms"] = round(_median_ms(call((0, T), (0, B), append=False), stream, steps), 5)
            res["decode_ratio_ours_over_fa4"] = round(res["decode_attention_ms"] / ours_phase_ms["decode"], 4)
    except Exception as e:  # noqa: BLE001
        res["unavailable"] = f"FA4 call failed: {e!r}"[:400]
    torch.cuda.synchronize(dev)
    return res


# ----------------------------------------------------------------------------
# multi-GPU in-run check
# ----------------------------------------------------------------------------
def check_gathered(arm: Arm, nseq: int = 4) -> dict:
    """Sampled rows of the gathered [B, Hq, 128] output against a torch fp32
    attention over the same pages: every rank computes its own heads' rows,
    the rows are all-gathered (outside the timed region) and every rank
    compares all heads of its gathered output.  Tolerances: bf16 max-abs
    2e-2, mean-abs 2e-3."""
    import torch.distributed as dist

    b = arm.batch
    B, bs = arm.B, arm.kc.shape[1]
    seqs = sorted({0, B // 3, (2 * B) // 3, B - 1})[:nseq]
    grp = arm.hq // arm.hkv
    refs = []
    for s in seqs:
        L = int(b.seq_lens[s])
        npg = (L + bs - 1) // bs
        blocks = b.block_table[s, :npg].long()
        k = arm.kc[blocks].reshape(npg * bs, arm.hkv, 128)[:L].float()
        v = arm.vc[blocks].reshape(npg * bs, arm.hkv, 128)[:L].float()
        q = b.q[s].float().view(arm.hkv, grp, 128)
        sc = torch.einsum("hgd,lhd->hgl", q, k) * b.softmax_scale
        p = torch.softmax(sc, dim=-1)
        refs.append(torch.einsum("hgl,lhd->hgd", p, v).reshape(arm.hq, 128))
    ref = torch.stack(refs)  # [n, hq_local, 128]
    allref = torch.empty(arm.world, *ref.shape, dtype=ref.dtype, device=ref.device)
    dist.all_gather_into_tensor(allref, ref)
    want = allref.permute(1, 0, 2, 3).reshape(len(seqs), arm.hq * arm.world, 128)
    got = arm.full_out[seqs].float()
    err = (got - want).abs()
    mx = _all_max(float(err.max()), arm.world, arm.dev)
    mean = _all_max(float(err.mean()), arm.world, arm.dev)
    return {"seqs": seqs, "heads": arm.hq * arm.world, "max_abs": mx, "mean_abs": mean,
            "ok": bool(mx <= 2e-2 and mean <= 2e-3),
            "reference": "torch fp32 attention over the gathered pages, every rank's heads all-gathered"}


def time_local_decode(arm: Arm, n: int = 20) -> float:
    """KV-head-sharded runs with the gather fused in: this rank's decode alone
    (the plain kernel over the same shard and inputs, into a scratch output),
    ``n`` launches back to back with CUDA events at the ends; max over ranks.
    The fused step minus this is what the exchange costs."""
    from ps_attn import ops

    b, scale = arm.batch, arm.batch.softmax_scale
    scratch = torch.empty(arm.B, arm.hq, 128, dtype=b.q.dtype, device=arm.dev)
    kw = dict(query_start_loc=b.query_start_loc, workspace=arm.ws, **arm.skw)

    def run():
        ops.paged_decode(b.q, arm.kc, arm.vc, b.block_table, b.seq_lens, scale, scratch, **kw)

    with torch.cuda.stream(arm.stream):
        for _ in range(3):
            run()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(arm.stream)
        for _ in range(n):
            run()
        e1.record(arm.stream)
    e1.synchronize()
    return _all_max(e0.elapsed_time(e1) / n, arm.world, arm.dev)


# ----------------------------------------------------------------------------
# end to end through the public ops
# ----------------------------------------------------------------------------
def run_e2e(arm: Arm, steps: int) -> dict:
    """The step as a serving engine runs it: this step's inputs copied from
    pinned host memory into persistent device buffers, the step's ops
    replayed from CUDA graphs captured over those buffers (what vLLM does
    for decode), and the whole attention output read back to the host.
    KV-head-sharded runs include the head all-gather."""
    b = arm.batch
    # the step's inputs packed into one pinned staging buffer (256-byte
    # aligned pieces) and one device buffer of the same layout: a single
    # host-to-device copy per step, as an engine stages its step inputs
    offs, total = {}, 0
    for k in INPUT_KEYS:
        t = getattr(b, k)
        offs[k] = total
        total += (t.numel() * t.element_size() + 255) // 256 * 256
    host_buf = torch.empty(total, dtype=torch.uint8).pin_memory()
    dev_buf = torch.empty(total, dtype=torch.uint8, device=arm.dev)

    def view(buf, k):
        t = getattr(b, k)
        n = t.numel() * t.element_size()
        return buf[offs[k]:offs[k] + n].view(t.dtype).view(t.shape)

    for k in INPUT_KEYS:
        view(host_buf, k).copy_(getattr(b, k).cpu())
    dev_in = {k: view(dev_buf, k) for k in INPUT_KEYS}
    dev_buf.copy_(host_buf)
    result = arm.result()
    out_host = torch.empty(result.shape, dtype=result.dtype).pin_memory()
    h2d = sum(getattr(b, k).numel() * getattr(b, k).element_size() for k in INPUT_KEYS)
    d2h = result.numel() * result.element_size()
    ops_ = [fn for _, fn in arm.phases(dev_in)]
    stream = arm.stream
    graphs = []

    def eager():
        dev_buf.copy_(host_buf, non_blocking=True)
        for fn in ops_:
            fn()
        out_host.copy_(result, non_blocking=True)

    with torch.cuda.stream(stream):
        for _ in range(3):
            eager()
        stream.synchronize()
        if arm.use_graph:
            # the copies and the ops of a step in one graph (memcpy nodes from
            # and to the pinned buffers): one launch per step
            step_graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(step_graph, stream=stream):
                eager()
            graphs.append(step_graph)
    one = graphs[0].replay if graphs else eager

    with torch.cuda.stream(stream):
        for _ in range(3):
            one()
    torch.cuda.synchronize(arm.dev)
    if arm.world > 1:
        import torch.distributed as dist

        dist.barrier()
    a = torch.cuda.Event(enable_timing=True)
    e = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        a.record(stream)
        for _ in range(steps):
            one()
        e.record(stream)
    torch.cuda.synchronize(arm.dev)
    ms = _all_max(a.elapsed_time(e) / steps, arm.world, arm.dev)
    graphs.clear()  # before any process-group teardown (a graph may hold NCCL calls)
    replicas = 1 if arm.sharded else arm.world
    return {"value": round(b.num_tokens * replicas / (ms / 1e3), 1), "unit": "tokens/s",
            "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
            "ms_per_step": round(ms, 5), "steps": steps, "cuda_graph": arm.use_graph,
            "note": "per step: the step's inputs (q, k, v, slots, lengths, block table, query starts) in one "
                    "pinned buffer -> device, the ops, the whole output -> pinned host; copies and ops replayed "
                    "from one CUDA graph per step"}


# ----------------------------------------------------------------------------
# side configs (N = 1): 2, 3, 4 with the FA4 bar
# ----------------------------------------------------------------------------
def side_config(cfg: int, dev, steps: int, warmup: int, fa4: bool) -> dict:
    arm = Arm(cfg, dev)
    arm.setup()
    t = arm.time(steps, warmup)
    ms = t["ms"]
    res = {"workload": CONFIG_NAMES[cfg], "tokens_per_s": round(arm.batch.num_tokens / (ms / 1e3), 1),
           "ms_per_step": round(ms, 5), "phase_ms": {k: round(v, 5) for k, v in t["phase_ms"].items()},
           "decode": decode_roofline(arm, t["phase_ms"]["decode"], profile_traffic(f"paged_decode_cfg{cfg}"))}
    if cfg == 3:
        res["decode"]["note"] = "bytes count each shared prefix page once (unique pages)"
    if arm.mixed:
        res["prefill"] = prefill_roofline(arm, t["phase_ms"]["prefill"])
    if fa4:
        res["fa4"] = fa4_compare(arm, steps, ms, t["phase_ms"])
    arm.close()
    del arm
    torch.cuda.empty_cache()
    return res


def run_ours(args):
    from ps_attn import _lib, workloads

    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    _lib.load(build_if_stale=False)
    cfg = args.config
    arm = Arm(cfg, dev, world, rank, kv_fp8=args.kv_fp8, cascade=args.cascade, fused=not args.unfused,
              gather=args.gather, use_graph=not args.no_graph, max_seqs=args.max_seqs)
    arm.setup()
    sampler = None if args.quick else ClockSampler(local)
    t = arm.time(args.steps, args.warmup, sampler)
    ms = t["ms"]
    pm = t["phase_ms"]
    check = check_gathered(arm) if arm.sharded else None
    alone_ms = time_local_decode(arm) if arm.sharded and arm.gather_kind == "fused" else None
    e2e = None if args.quick else run_e2e(arm, args.steps)

    tokens = arm.batch.num_tokens  # every rank produces all tokens (its heads when sharded)
    value = tokens * (1 if arm.sharded else world) / (ms / 1e3)
    step_bytes = workloads.hbm_bytes(arm.batch)
    # DRAM bytes of a full launch from the committed ncu summary (none for a
    # profiling subset or a KV-head shard, whose launches are smaller)
    traffic = (None if arm.sharded or args.max_seqs is not None
               else profile_traffic(f"paged_decode_{'fp8_' if args.kv_fp8 else ''}cfg{cfg}"))
    res = {
        "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 5),
        "higher_is_better": True, "scaling": "strong" if arm.sharded else "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": config_dict(cfg, args.max_seqs),
        "setup": {
            "parallelism": (f"kv-head tp{world} + " + {
                "fused": "head all-gather fused into the decode over NVLink peer memory "
                         "(ps_paged_decode_head_gather)",
                "peer": "NVLink peer-memory head gather (ps_head_gather)",
                "nccl": "NCCL all-gather"}[arm.gather_kind] if arm.sharded else
                            (f"batch replicas x{world}" if world > 1 else "single GPU")),
            "heads_this_gpu": {"q": arm.hq, "kv": arm.hkv},
            "kv_pool_bytes_this_gpu": arm.batch.kv_cache.numel() * arm.batch.kv_cache.element_size(),
            "l2": "inputs larger than L2 (KV pool > 126 MB); no flush",
            "cuda_graph": arm.use_graph,
            "kv_cache_dtype": "fp8_e4m3 (per-tensor scale)" if args.kv_fp8 else "bf16",
            "append_fused_into_decode": arm.fused,
            "cascade": arm.cascade,
        },
        "gpu_launches": arm.launches_per_step() * args.steps,
        "phase_ms": {k: round(v, 5) for k, v in pm.items()},
        "hbm_gbs_step": round(step_bytes / (ms / 1e3) / 1e9, 1),
        "hbm_frac_of_8tbs_step": round(step_bytes / (ms / 1e3) / 1e9 / NOMINAL_HBM_GBS, 4),
        "roofline": decode_roofline(arm, pm["decode"], traffic),
        "prefill": prefill_roofline(arm, pm["prefill"]) if arm.mixed else None,
        "e2e": e2e,
        "clocks": t["clocks"],
    }
    if arm.sharded:
        rx = (world - 1) * arm.B * arm.hq * 128 * arm.batch.q.element_size()
        if arm.gather_kind == "fused":
            extra = ms - alone_ms
            res["gather"] = {"kind": "fused into the decode launch (ps_paged_decode_head_gather)",
                             "ms_per_step": round(extra, 5), "share_of_step": round(extra / ms, 4),
                             "decode_alone_ms": round(alone_ms, 5), "bytes_received_per_gpu": rx,
                             "note": "rows stored into the peers over NVLink as the decode finishes them; "
                                     "ms_per_step = the fused step minus this rank's decode alone (the plain "
                                     "kernel on the same shard, timed back to back after the run, max over ranks)"}
        else:
            res["gather"] = {"kind": arm.gather_kind, "ms_per_step": round(pm["gather"], 5),
                             "share_of_step": round(pm["gather"] / ms, 4), "bytes_received_per_gpu": rx}
        res["check"] = check
    if arm.cascade:
        res["cascade"] = {"groups": int(arm.plan.views()["num_groups"].item()),
                          "note": "shared prompt pages read once per 16-column pass; plan built every step; "
                                  "roofline bytes count each shared page once"}
    if world == 1 and not args.quick:
        if not args.no_fa4 and not args.kv_fp8 and not arm.cascade and arm.fused:
            res["fa4"] = fa4_compare(arm, args.steps, ms, pm)
        if rank == 0:
            res["cpu_baseline"] = cpu_baseline(cfg, budget_s=args.cpu_budget)
    if (world == 1 and not args.quick and not args.no_side and cfg == DEFAULT_CONFIG and not args.kv_fp8
            and args.max_seqs is None):
        arm.close()
        del arm
        torch.cuda.empty_cache()
        side = {}
        for c in (2, 3, 4):
            side[f"cfg{c}"] = side_config(c, dev, args.steps, args.warmup, not args.no_fa4)
        res["configs"] = side
        res["prefill"] = side["cfg4"].get("prefill")
        if "fa4" in side["cfg4"] and "prefill_attention_ms" in side["cfg4"]["fa4"]:
            res["prefill"] = dict(res["prefill"], fa4_ms=side["cfg4"]["fa4"]["prefill_attention_ms"],
                                  ratio_ours_over_fa4=side["cfg4"]["fa4"]["prefill_ratio_ours_over_fa4"])
    if rank == 0:
        print(json.dumps(res), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()  # no peer still reads this rank's slab
        arm.close()
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
    elapsed_ms = _all_max(elapsed_ms, world, dev)
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
    e2e_ms = _all_max(e0.elapsed_time(e1), world, dev)
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
        "config": config_dict(cfg),
        "setup": {"mode": "decode context parallel", "kv_tokens_this_rank": batch.unique_tokens,
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
        q0, q1 = int(batch.query_start_loc[b]), int(batch.query_start_loc[b + 1])
        q = batch.q[q0:q1].float()
        o, _, lse = attention_ref(q[None], k[None], v[None], causal=True, return_lse=True)
        outs.append(o)
    return outs


def cpu_baseline(cfg, budget_s=20.0, steps=None, warmup=1):
    """Time the reference CPU step on a bounded sample of the workload: a
    seeded prefix subset of the sequences (all 64 for config 2), repeated
    until the time budget or ``steps`` is reached; tokens/s = new tokens
    processed / time."""
    from ps_attn import workloads

    attention_ref = load_reference_attention()
    kind = "reference"
    if attention_ref is None:  # vLLM missing: the oracle port stands in
        from oracle import ps_oracle

        kind = "port"

        def attention_ref(q, k, v, causal=True, return_lse=True):
            o, l = ps_oracle.attention_ref(q[0].numpy(), k[0].numpy(), v[0].numpy(), causal=causal)
            return torch.from_numpy(o)[None], None, torch.from_numpy(l)[None]

    sub = {2: 64, 3: 16, 4: 16, 5: 16}[cfg]
    batch = workloads.make_config(cfg, device="cpu", max_seqs=sub)
    seqs = list(range(batch.num_seqs))
    toks = int(batch.num_tokens)
    for _ in range(warmup):
        reference_step(batch, attention_ref, seqs[:2])
    t_used = 0.0
    step_times = []
    while t_used < budget_s and (steps is None or len(step_times) < steps):
        t = time.perf_counter()
        reference_step(batch, attention_ref, seqs)
        dt = time.perf_counter() - t
        step_times.append(dt)
        t_used += dt
        if steps is None and len(step_times) >= 200:
            break
    value = toks * len(step_times) / t_used
    full = len(workloads.config_lengths(cfg)[1])
    return {"value": round(value, 2), "unit": "tokens/s", "cores": torch.get_num_threads(),
            "kind": kind,
            "sample": f"cfg{cfg}: {len(seqs)} of {full} sequences ({toks} new tokens) x {len(step_times)} steps "
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
        "ms_per_step": cb["ms_per_step"], "higher_is_better": True,
        "scaling": "strong" if args.config == 5 and world > 1 else "weak",
        "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
        "config": config_dict(args.config),
        "cpu_baseline": cb,
        "e2e": {"value": cb["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(res), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--config", type=int, default=DEFAULT_CONFIG, choices=[2, 3, 4, 5])
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--unfused", action="store_true",
                    help="separate append launch instead of the append fused into decode")
    ap.add_argument("--cascade", action="store_true",
                    help="config 3: shared-prefix (cascade) decode with a per-step plan")
    ap.add_argument("--dcp", action="store_true",
                    help="config 5 under decode context parallelism (tokens sharded, not heads)")
    ap.add_argument("--gather", default="fused", choices=["fused", "nccl", "peer"],
                    help="config 5 on N GPUs: head outputs stored into the peers by the decode itself "
                         "(fused), pulled over peer memory by a separate launch (peer), or all-gathered by NCCL")
    ap.add_argument("--kv-fp8", action="store_true",
                    help="decode configs over an fp8 (e4m3) KV cache, fused quantizing append")
    ap.add_argument("--interleave", type=int, default=1,
                    help="DCP: consecutive positions per rank (vLLM cp_kv_cache_interleave_size)")
    ap.add_argument("--cpu-budget", type=float, default=15.0)
    ap.add_argument("--no-fa4", action="store_true", help="skip the vLLM FA4 comparison")
    ap.add_argument("--no-side", action="store_true", help="N=1: skip configs 2-4 after the headline")
    ap.add_argument("--max-seqs", type=int, default=None,
                    help="profiling: a seeded prefix subset of the config's sequences (not a benchmark line)")
    ap.add_argument("--quick", action="store_true",
                    help="timed steps only: no end-to-end, CPU baseline, FA4, side configs or clock sampling")
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
