"""Shared test helpers: golden fixtures, oracle evaluation, tolerance checks.

Tolerances (from the benchmark spec): append and page gathers bit-exact; bf16
attention output within max-abs 2e-2 and mean-abs 2e-3 of the fp32 reference;
LSE within 1e-3.
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import torch

from oracle import ps_oracle
from ps_attn import workloads

GOLDEN = Path(__file__).resolve().parent / "golden"
OUT_MAX_ABS = 2e-2
OUT_MEAN_ABS = 2e-3
LSE_ABS = 1e-3


def golden_meta():
    return json.loads((GOLDEN / "golden_meta.json").read_text())


def build_case(spec, dtype=torch.bfloat16, device="cpu"):
    spec = dict(spec)
    if "cfg" in spec:
        return workloads.make_config(spec["cfg"], device=device)
    spec.setdefault("dtype", dtype)
    return workloads.make_batch(device=device, **spec)


def checksum(batch):
    parts = [batch.q, batch.key, batch.value, batch.kv_cache]
    return float(sum(p.double().sum().item() for p in parts))


def load_attn_golden(name):
    d = np.load(GOLDEN / f"attn_{name}.npz")
    return d["out"], d["lse"]


def to_np32(t: torch.Tensor) -> np.ndarray:
    return t.detach().to("cpu", torch.float32).numpy()


def oracle_append(batch):
    """Oracle append on a CPU copy of ``batch``'s cache: (key_cache, value_cache)."""
    kc = batch.kv_cache[0].detach().cpu().clone()
    vc = batch.kv_cache[1].detach().cpu().clone()
    # byte-level append on numpy views keeps bf16 bit patterns intact
    view = (lambda t: t.view(torch.int16).numpy()) if kc.dtype == torch.bfloat16 else (lambda t: t.numpy())
    ps_oracle.kv_append(view(batch.key.cpu()), view(batch.value.cpu()), view(kc), view(vc),
                        batch.slot_mapping.cpu().numpy())
    return kc, vc


def oracle_step(batch, causal=True):
    """Oracle append + paged attention on a CPU copy of ``batch``.

    Returns (key_cache, value_cache) after the append (torch, original dtype)
    and (out fp32 [T,Hq,D], lse fp32 [Hq,T]).
    """
    kc, vc = oracle_append(batch)
    out, lse = ps_oracle.paged_attention(
        to_np32(batch.q), to_np32(kc), to_np32(vc), batch.block_table.cpu().numpy(),
        batch.seq_lens.cpu().numpy(), batch.query_start_loc.cpu().numpy(),
        batch.softmax_scale, causal=causal)
    return (kc, vc), (out, lse)


def assert_attn_close(out, ref_out, lse=None, ref_lse=None, rows=None,
                      max_abs=OUT_MAX_ABS, mean_abs=OUT_MEAN_ABS, lse_abs=LSE_ABS):
    out = np.asarray(out, dtype=np.float32)
    ref_out = np.asarray(ref_out, dtype=np.float32)
    if rows is not None:
        out, ref_out = out[rows], ref_out[rows]
    assert np.isfinite(out).all(), "non-finite output"
    err = np.abs(out - ref_out)
    assert err.max(initial=0.0) <= max_abs, f"max abs err {err.max():.3e} > {max_abs}"
    assert err.mean() <= mean_abs if err.size else True, f"mean abs err {err.mean():.3e} > {mean_abs}"
    if lse is not None:
        lse = np.asarray(lse, dtype=np.float32)
        ref_lse = np.asarray(ref_lse, dtype=np.float32)
        if rows is not None:
            lse, ref_lse = lse[:, rows], ref_lse[:, rows]
        both_inf = np.isneginf(lse) & np.isneginf(ref_lse)
        assert (np.isneginf(lse) == np.isneginf(ref_lse)).all(), "LSE -inf pattern differs"
        d = np.abs(np.where(both_inf, 0.0, lse - ref_lse))
        assert d.max(initial=0.0) <= lse_abs, f"LSE err {d.max():.3e} > {lse_abs}"
