"""CPU: the rotary-embedding restatement against vLLM's own torch-native
RoPE (golden vectors from ``RotaryEmbedding.forward_static``): bit-exact."""
from __future__ import annotations

import numpy as np
import pytest

from helpers import GOLDEN, golden_meta
from oracle import ps_oracle

CASES = sorted(golden_meta()["rope"])


def as_f32(a, dtype):
    if dtype == "bf16":
        return (a.astype(np.uint16).astype(np.uint32) << 16).view(np.float32)
    return a.astype(np.float32)


def load(name):
    m = golden_meta()["rope"][name]
    d = dict(np.load(GOLDEN / f"rope_{name}.npz"))
    dt = "bf16" if "bfloat16" in m["dtype"] else "fp16"
    cdt = "bf16" if "bfloat16" in m["cache_dtype"] else ("fp16" if "float16" in m["cache_dtype"] else "fp32")
    T, Hq, Hkv, D, rot, neox = (int(v) for v in d["shape"])
    return m, d, dt, cdt, (T, Hq, Hkv, D, rot, bool(neox))


@pytest.mark.parametrize("name", CASES)
def test_rope_oracle_matches_reference_golden(name):
    m, d, dt, cdt, (T, Hq, Hkv, D, rot, neox) = load(name)
    rows = as_f32(d["cos_sin_rows"], cdt)
    for x_in, x_out, H in (("q_in", "q_out", Hq), ("k_in", "k_out", Hkv)):
        x = as_f32(d[x_in], dt).reshape(T, H, D)
        got = ps_oracle.rope(x, d["positions"], rows, rot, neox, dt)
        want = as_f32(d[x_out], dt).reshape(T, H, D)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), name


def test_bf16_rounding_is_nearest_even():
    x = np.array([1.0, 1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, 1.0 + 2 ** -9, -2.5, 0.0], dtype=np.float32)
    r = ps_oracle.round_to(x, "bf16")
    assert r.tolist() == [1.0, 1.0, 1.0 + 2 ** -6, 1.0, -2.5, 0.0]
