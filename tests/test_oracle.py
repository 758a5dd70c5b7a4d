"""CPU: pin the oracle against the reference's own outputs (golden vectors)."""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from helpers import (GOLDEN, assert_attn_close, build_case, checksum, golden_meta,
                     load_attn_golden, oracle_step)
from oracle import ps_oracle

META = golden_meta()


@pytest.mark.parametrize("name", sorted(META["attention"]))
def test_oracle_matches_attention_ref_golden(name):
    spec = META["attention"][name]["spec"]
    batch = build_case(spec)
    cs = checksum(batch)
    assert math.isclose(cs, META["attention"][name]["input_checksum"], rel_tol=1e-9, abs_tol=1e-6), \
        "input generator drifted from the one the goldens were made with"
    _, (out, lse) = oracle_step(batch)
    gout, glse = load_attn_golden(name)
    # the oracle restates attention_ref in fp32: agreement to fp32 rounding
    np.testing.assert_allclose(out, gout, atol=2e-5, rtol=0)
    fin = np.isfinite(glse)
    assert (np.isfinite(lse) == fin).all()
    np.testing.assert_allclose(lse[fin], glse[fin], atol=2e-5, rtol=0)


@pytest.mark.parametrize("name", ["bf16", "fp32"])
def test_oracle_append_matches_triton_golden(name):
    d = np.load(GOLDEN / f"append_{name}.npz")
    qkv = d["qkv"]
    H, D = d["key_cache_in"].shape[2:]
    T = len(d["slot_mapping"])
    key = qkv[:, 4 * D:(4 + H) * D].reshape(qkv.shape[0], H, D)
    value = qkv[:, (4 + H) * D:].reshape(qkv.shape[0], H, D)
    kc, vc = d["key_cache_in"].copy(), d["value_cache_in"].copy()
    assert key.shape[0] > T  # padded rows beyond slot_mapping must be ignored
    ps_oracle.kv_append(key, value, kc, vc, d["slot_mapping"])
    assert np.array_equal(kc.view(np.uint8), d["key_cache_out"].view(np.uint8))
    assert np.array_equal(vc.view(np.uint8), d["value_cache_out"].view(np.uint8))


def test_gather_pages_addressing():
    cache = np.arange(5 * 16 * 2 * 4, dtype=np.float32).reshape(5, 16, 2, 4)
    bt = np.array([3, 0, 4])
    rows = ps_oracle.gather_pages(cache, bt, 35)
    assert rows.shape == (35, 2, 4)
    assert np.array_equal(rows[:16], cache[3])
    assert np.array_equal(rows[16:32], cache[0])
    assert np.array_equal(rows[32:], cache[4, :3])
    assert ps_oracle.gather_pages(cache, bt, 0).shape[0] == 0


@pytest.mark.parametrize("nsplit", [1, 2, 3, 7])
def test_split_then_combine_equals_unsplit(nsplit):
    rng = np.random.default_rng(nsplit)
    L, hq, hkv, d = 203, 8, 2, 128
    q = rng.standard_normal((hq, d)).astype(np.float32)
    k = rng.standard_normal((L, hkv, d)).astype(np.float32)
    v = rng.standard_normal((L, hkv, d)).astype(np.float32)
    cuts = np.linspace(0, L, nsplit + 1).astype(int)
    splits = list(zip(cuts[:-1], cuts[1:]))
    o_s, lse_s = ps_oracle.split_partials(q, k, v, splits, 1 / math.sqrt(d))
    o, lse = ps_oracle.combine(o_s, lse_s)
    ro, rlse = ps_oracle.attention_ref(q[None], k, v, causal=False)
    np.testing.assert_allclose(o, ro[0], atol=1e-5)
    np.testing.assert_allclose(lse, rlse[:, 0], atol=1e-5)


def test_combine_empty_splits_and_all_empty():
    d = 4
    o_s = np.zeros((3, 2, d), np.float32)
    lse_s = np.full((3, 2), -np.inf, np.float32)
    o_s[1, 0] = 1.5
    lse_s[1, 0] = 0.25  # row 0: a single non-empty split among empties
    o, lse = ps_oracle.combine(o_s, lse_s)
    np.testing.assert_allclose(o[0], 1.5)
    assert lse[0] == pytest.approx(0.25, abs=1e-6)
    assert (o[1] == 0).all() and np.isneginf(lse[1])  # row 1: every split empty


def test_attention_ref_causal_bottom_right_and_empty():
    rng = np.random.default_rng(0)
    q = rng.standard_normal((3, 2, 8)).astype(np.float32)
    k = rng.standard_normal((5, 1, 8)).astype(np.float32)
    v = rng.standard_normal((5, 1, 8)).astype(np.float32)
    out, lse = ps_oracle.attention_ref(q, k, v, causal=True)
    # last query row sees all keys; first sees keys 0..2
    full, _ = ps_oracle.attention_ref(q[2:], k, v, causal=False)
    np.testing.assert_allclose(out[2], full[0], atol=1e-6)
    first, _ = ps_oracle.attention_ref(q[:1], k[:3], v[:3], causal=False)
    np.testing.assert_allclose(out[0], first[0], atol=1e-6)
    eo, el = ps_oracle.attention_ref(q[:1], k[:0], v[:0])
    assert (eo == 0).all() and np.isneginf(el).all()


def test_num_splits_heuristic():
    assert ps_oracle.num_splits_heuristic(4, 148, 4, 128) == 1
    assert ps_oracle.num_splits_heuristic(4, 148, 100, 128) == 37
    assert ps_oracle.num_splits_heuristic(1, 148, 200, 128) == 128


def test_decode_slots_match_workload():
    b = build_case(dict(q_lens=[1, 1], seq_lens=[17, 3], num_q_heads=2, num_kv_heads=1, seed=3))
    slots = ps_oracle.decode_slots(b.block_table.numpy(), b.seq_lens.numpy(), 16)
    assert np.array_equal(slots, b.slot_mapping.numpy())
