"""CPU: the torch.library registration of the C ABI (``torch.ops.ps_attn.*``):
schemas declare exactly the mutated arguments, and the fake implementations
trace shapes under FakeTensorMode without launching anything."""
from __future__ import annotations

import pytest
import torch

from ps_attn import torch_ops  # noqa: F401  (registers the operators)


def _schema(name):
    return str(getattr(torch.ops.ps_attn, name).default._schema)


def _mutated(schema):
    return {a.name for a in schema.arguments if a.alias_info is not None and a.alias_info.is_write}


def test_schemas_declare_mutations():
    op = torch.ops.ps_attn
    assert _mutated(op.kv_append.default._schema) == {"key_cache", "value_cache"}
    assert _mutated(op.paged_decode.default._schema) == {"key_cache", "value_cache", "out", "lse", "workspace"}
    assert _mutated(op.chunked_prefill.default._schema) == {"out", "lse", "workspace"}
    s = _schema("paged_decode")
    assert "Tensor? new_key" in s and "float softmax_scale" in s and "SymInt max_seq_len" in s
    assert "Tensor? query_start_loc" in s and s.endswith("-> ()")
    assert "Tensor query_start_loc" in _schema("chunked_prefill")


def test_fake_implementations_trace_without_a_gpu():
    from torch._subclasses.fake_tensor import FakeTensorMode

    with FakeTensorMode():
        T, hq, hkv, d, nb = 4, 16, 8, 128, 64
        q = torch.empty(T, hq, d, dtype=torch.bfloat16)
        kc = torch.empty(nb, 16, hkv, d, dtype=torch.bfloat16)
        vc = torch.empty_like(kc)
        bt = torch.zeros(T, 8, dtype=torch.int32)
        sl = torch.full((T,), 100, dtype=torch.int32)
        qsl = torch.arange(T + 1, dtype=torch.int32)
        out = torch.empty_like(q)
        lse = torch.empty(hq, T)
        ws = torch.empty(1 << 20, dtype=torch.uint8)
        slots = torch.arange(T, dtype=torch.int64)
        k = torch.empty(T, hkv, d, dtype=torch.bfloat16)
        torch.ops.ps_attn.kv_append(k, k, kc, vc, slots)
        torch.ops.ps_attn.paged_decode(q, kc, vc, bt, sl, qsl, 0.088, 100, out, lse, ws, k, k, slots)
        torch.ops.ps_attn.chunked_prefill(q, kc, vc, bt, sl, qsl, 0.088, 100, out, lse, ws)
        assert out.shape == (T, hq, d)


def test_workspace_view_rejects_other_dtypes():
    with pytest.raises(ValueError):
        torch_ops._WorkspaceView(torch.zeros(16, dtype=torch.int32), 1)
