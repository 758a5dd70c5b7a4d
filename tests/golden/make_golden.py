"""Generate the golden vectors in this directory from the reference's own code.

Run in a container where vLLM 0.22 is installed (not needed at test time):

    python tests/golden/make_golden.py

* Attention: vLLM's FA4 torch reference ``attention_ref``
  (``vllm/vllm_flash_attn/cute/testing.py:326-455``), loaded by file path
  because importing the ``vllm.vllm_flash_attn`` package needs its CUDA
  extensions.  It is evaluated in fp32 (inputs upcast first) on the pages each
  sequence's block table names, with ``causal=True`` as
  ``flash_attn.py:796-817`` passes it.
* KV append: vLLM's Triton kernel ``reshape_and_cache_kernel_flash``
  (``vllm/v1/attention/ops/triton_reshape_and_cache_flash.py:17-124``) run on CPU
  tensors under the Triton interpreter (``TRITON_INTERPRET=1``).

* Rotary embedding (for the fused RoPE + KV append): vLLM's
  ``RotaryEmbedding.forward_static``
  (``vllm/model_executor/layers/rotary_embedding/base.py:140-181``, the
  torch-native path ``forward_native`` takes) on CPU tensors, neox and GPT-J
  styles, full and partial rotary dims, bf16 and fp16, with the cos/sin cache
  in the model dtype or in fp32.  The inputs are stored with the outputs
  (``rope_*.npz``); only the cos/sin rows at the tested positions are stored.
  ``python tests/golden/make_golden.py --only rope`` regenerates just these.

* Decode context parallelism (``dcp_*.npz``): vLLM's Triton slot-mapping
  kernel ``_compute_slot_mapping_kernel`` (``vllm/v1/worker/block_table.py:326-380``)
  for several (world, interleave, rank), and the LSE correction + merge of
  the DCP decode: ``correct_attn_out`` (``vllm/v1/attention/ops/common.py:99-170``,
  Triton kernel ``_correct_attn_cp_out_kernel``) on every rank's partial,
  the sum over ranks (what ``reduce_scatter`` computes), then the Triton
  ``merge_attn_states`` (``triton_merge_attn_states.py:14-140``) with the new
  tokens' own attention -- all under the interpreter, on inputs that include
  empty slices (LSE -inf), FA2's +inf and NaN LSEs.
  ``python tests/golden/make_golden.py --only dcp`` regenerates just these.

Inputs are regenerated at test time from the seeds recorded here by
``ps_attn.workloads.make_batch`` (CPU generator); a checksum of the inputs is
stored so a generator change is detected instead of silently comparing
different data.
"""
from __future__ import annotations

import importlib.util
import json
import os
import sys
from pathlib import Path

os.environ.setdefault("TRITON_INTERPRET", "1")

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO / "prime-rl_b200"))

from ps_attn import workloads  # noqa: E402

VLLM = Path(importlib.util.find_spec("vllm").origin).parent


def load_attention_ref():
    path = VLLM / "vllm_flash_attn" / "cute" / "testing.py"
    spec = importlib.util.spec_from_file_location("fa4_testing_ref", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.attention_ref


# (name, make_batch kwargs) -- every attention case applies the append first
ATTN_CASES = {
    "cfg1": dict(cfg=1),
    "gqa1": dict(q_lens=[1, 1, 1], seq_lens=[1, 17, 100], num_q_heads=2, num_kv_heads=2, seed=11),
    "gqa2": dict(q_lens=[1, 1, 1, 1], seq_lens=[16, 33, 250, 64], num_q_heads=4, num_kv_heads=2, seed=12),
    "gqa4": dict(q_lens=[1, 1], seq_lens=[47, 300], num_q_heads=8, num_kv_heads=2, seed=13),
    "gqa8": dict(q_lens=[1, 1, 1], seq_lens=[129, 5, 512], num_q_heads=16, num_kv_heads=2, seed=14),
    "gqa16": dict(q_lens=[1, 1], seq_lens=[80, 31], num_q_heads=16, num_kv_heads=1, seed=15),
    "bs32": dict(q_lens=[1, 1, 1], seq_lens=[70, 32, 200], num_q_heads=8, num_kv_heads=2,
                 block_size=32, seed=16),
    "prefill": dict(q_lens=[5, 37, 1, 16], seq_lens=[5, 90, 33, 200], num_q_heads=8,
                    num_kv_heads=2, seed=17),
    "grpo": dict(q_lens=[1] * 8, seq_lens=[70, 80, 65, 99, 64 + 1, 130, 77, 66], num_q_heads=8,
                 num_kv_heads=2, share_groups=4, shared_prefix_tokens=64, seed=18),
}


def build_case(spec, dtype=torch.bfloat16):
    spec = dict(spec)
    if "cfg" in spec:
        return workloads.make_config(spec["cfg"], device="cpu")
    spec.setdefault("dtype", dtype)
    return workloads.make_batch(device="cpu", **spec)


def checksum(batch):
    parts = [batch.q, batch.key, batch.value, batch.kv_cache]
    return float(sum(p.double().sum().item() for p in parts))


def torch_append(batch):
    """Index-put append used to prepare the cache for the attention goldens."""
    kc, vc = batch.kv_cache[0], batch.kv_cache[1]
    nb, bs, h, d = kc.shape
    ok = batch.slot_mapping >= 0
    kc.view(-1, h, d)[batch.slot_mapping[ok]] = batch.key[ok]
    vc.view(-1, h, d)[batch.slot_mapping[ok]] = batch.value[ok]


def attention_golden(name, spec, attention_ref):
    batch = build_case(spec)
    cs = checksum(batch)
    torch_append(batch)
    kc, vc = batch.kv_cache[0], batch.kv_cache[1]
    bs = kc.shape[1]
    T, hq, d = batch.q.shape
    out = torch.zeros(T, hq, d, dtype=torch.float32)
    lse = torch.full((hq, T), float("-inf"), dtype=torch.float32)
    qsl = batch.query_start_loc.tolist()
    for b, L in enumerate(batch.seq_lens.tolist()):
        t0, t1 = qsl[b], qsl[b + 1]
        if t1 <= t0:
            continue
        npg = (L + bs - 1) // bs
        blocks = batch.block_table[b, :npg].long()
        k = kc[blocks].reshape(npg * bs, *kc.shape[2:])[:L].float()
        v = vc[blocks].reshape(npg * bs, *vc.shape[2:])[:L].float()
        q = batch.q[t0:t1].float()
        o, _, l = attention_ref(q[None], k[None], v[None], causal=True, return_lse=True)
        out[t0:t1] = o[0]
        lse[:, t0:t1] = l[0]
    return dict(out=out.numpy(), lse=lse.numpy()), cs


def append_golden(triton_mod, dtype, seed):
    """Run vLLM's Triton append kernel under the interpreter on a small cache."""
    g = torch.Generator().manual_seed(seed)
    T, H, D, NB, bs = 9, 2, 128, 6, 16
    # key/value are views into a wider qkv row (token stride > H*D), like vLLM's
    qkv = torch.randn(T + 2, (4 + 2 * H) * D, generator=g).to(dtype)
    key = qkv[:, 4 * D:(4 + H) * D].view(T + 2, H, D)
    value = qkv[:, (4 + H) * D:].view(T + 2, H, D)
    kc = torch.randn(NB, bs, H, D, generator=g).to(dtype)
    vc = torch.randn(NB, bs, H, D, generator=g).to(dtype)
    kc0, vc0 = kc.clone(), vc.clone()
    slots = torch.tensor([3, -1, 17, 40, 95, 0, -1, 64, 33], dtype=torch.int64)
    n = H * D
    run_dtype = torch.int16 if dtype == torch.bfloat16 else dtype
    kc_r, vc_r = kc.view(run_dtype), vc.view(run_dtype)
    key_r, value_r = key.view(run_dtype), value.view(run_dtype)
    triton_mod.reshape_and_cache_kernel_flash[(T, 1)](
        key_r, value_r, kc_r, vc_r, slots, torch.ones(1), torch.ones(1),
        key_r.stride(0), value_r.stride(0), kc_r.stride(0), kc_r.stride(2), 0, 0, kc_r.stride(1),
        H, D, bs, 1, False, False, 256)
    as_np = (lambda t: t.view(torch.int16).numpy()) if dtype == torch.bfloat16 else (lambda t: t.numpy())
    return dict(qkv=as_np(qkv), key_cache_in=as_np(kc0), value_cache_in=as_np(vc0),
                slot_mapping=slots.numpy(), key_cache_out=as_np(kc), value_cache_out=as_np(vc))


ROPE_CASES = {
    # name: (dtype, cache dtype, rotary_dim, is_neox, seed)
    "bf16_neox": (torch.bfloat16, torch.bfloat16, 128, True, 31),
    "bf16_gptj": (torch.bfloat16, torch.bfloat16, 128, False, 32),
    "fp16_partial": (torch.float16, torch.float16, 64, True, 33),
    "bf16_fp32cache": (torch.bfloat16, torch.float32, 128, True, 34),
}
ROPE_MAX_POS = 40960   # Qwen3 max_position_embeddings
ROPE_THETA = 1.0e6     # Qwen3 rope_theta


def rope_golden(dtype, cache_dtype, rot, neox, seed):
    """vLLM's torch-native rotary embedding on random q/k rows."""
    from vllm.model_executor.layers.rotary_embedding.base import RotaryEmbedding

    g = torch.Generator().manual_seed(seed)
    T, Hq, Hkv, D = 9, 4, 2, 128
    positions = torch.tensor([0, 1, 7, 255, 1000, 4097, 20000, 40958, 40959], dtype=torch.int64)
    # the cache as vLLM's RotaryEmbedding._compute_cos_sin_cache builds it
    inv_freq = 1.0 / (ROPE_THETA ** (torch.arange(0, rot, 2, dtype=torch.float) / rot))
    freqs = torch.einsum("i,j -> ij", positions.to(torch.float), inv_freq)
    rows = torch.cat((freqs.cos(), freqs.sin()), dim=-1).to(cache_dtype)  # [T, rot]
    q = torch.randn(T, Hq * D, generator=g).to(dtype)
    k = torch.randn(T, Hkv * D, generator=g).to(dtype)
    full = torch.zeros(ROPE_MAX_POS, rot, dtype=cache_dtype)
    full[positions] = rows
    qo, ko = RotaryEmbedding.forward_static(positions, q.clone(), k.clone(), D, rot, full, neox)
    bits = (lambda t: t.view(torch.int16).numpy()) if dtype == torch.bfloat16 else (lambda t: t.numpy())
    cbits = (lambda t: t.view(torch.int16).numpy()) if cache_dtype == torch.bfloat16 else (lambda t: t.numpy())
    return dict(positions=positions.numpy(), cos_sin_rows=cbits(rows), q_in=bits(q), k_in=bits(k),
                q_out=bits(qo), k_out=bits(ko), shape=np.array([T, Hq, Hkv, D, rot, int(neox)]))


def main_rope(meta):
    meta["rope"] = {}
    for name, (dtype, cdtype, rot, neox, seed) in ROPE_CASES.items():
        np.savez_compressed(HERE / f"rope_{name}.npz", **rope_golden(dtype, cdtype, rot, neox, seed))
        meta["rope"][name] = {"dtype": str(dtype), "cache_dtype": str(cdtype), "rotary_dim": rot,
                              "is_neox": neox, "seed": seed, "max_position": ROPE_MAX_POS}
        print(f"rope_{name}: written")


DCP_SLOT_CASES = {
    # name: (world, interleave, seed)
    "w2_i1": (2, 1, 41),
    "w4_i1": (4, 1, 42),
    "w2_i4": (2, 4, 43),
    "w8_i16": (8, 16, 44),
    "w3_i2": (3, 2, 45),
}
DCP_COMBINE_CASES = {
    # name: (world, dtype of the partial outputs, seed).  fp32 only: the
    # Triton interpreter converts fp32 to bf16 by truncation where the GPU
    # rounds to nearest even, so bf16 stores would pin the interpreter.
    "w2_fp32": (2, torch.float32, 51),
    "w4_fp32": (4, torch.float32, 52),
}


def dcp_slot_golden(world, interleave, seed):
    """vLLM's slot mapping for every rank of a DCP group."""
    from vllm.v1.worker import block_table as btm

    g = torch.Generator().manual_seed(seed)
    B, P, bs = 3, 12, 16
    bt = torch.randperm(B * P + 7, generator=g)[:B * P].to(torch.int32).view(B, P)
    cap = P * bs * world  # positions a row of P virtual blocks covers
    counts = [5, 9, 14]
    qsl = torch.tensor([0] + list(np.cumsum(counts)), dtype=torch.int32)
    pos = torch.cat([torch.randint(0, cap, (c,), generator=g) for c in counts]).to(torch.int64)
    T = int(qsl[-1])
    slots = []
    for r in range(world):
        out = torch.full((T + 4,), -7, dtype=torch.int64)
        btm._compute_slot_mapping_kernel[(B + 1,)](
            T, T + 4, qsl, pos, bt, bt.stride(0), bs, out, TOTAL_CP_WORLD_SIZE=world,
            TOTAL_CP_RANK=r, CP_KV_CACHE_INTERLEAVE_SIZE=interleave, PAD_ID=-1, BLOCK_SIZE=1024)
        slots.append(out[:T].numpy())
    return dict(block_table=bt.numpy(), query_start_loc=qsl.numpy(), positions=pos.numpy(),
                slots=np.stack(slots), shape=np.array([world, interleave, bs]))


def dcp_combine_golden(world, dtype, seed):
    """correct_attn_out on every rank, the sum over ranks, merge_attn_states."""
    from vllm.v1.attention.ops import common as cm
    from vllm.v1.attention.ops import triton_merge_attn_states as tm

    g = torch.Generator().manual_seed(seed)
    T, H, D = 6, 4, 128
    o_r = torch.randn(world, T, H, D, generator=g).to(dtype)
    lse_r = (torch.randn(world, T, H, generator=g) * 3.0).float()  # [N, B, H] as cp_lse_* takes
    lse_r[1, 0, :] = -float("inf")   # rank 1 holds none of token 0's context
    o_r[1, 0] = 0
    lse_r[:, 1, :] = -float("inf")   # token 1: empty context on every rank
    o_r[:, 1] = 0
    lse_r[0, 2, 1] = float("inf")    # FA2's empty-sum convention
    lse_r[world - 1, 3, 2] = float("nan")
    s_out = torch.randn(T, H, D, generator=g).to(dtype)
    s_lse = (torch.randn(H, T, generator=g) * 3.0).float()
    corrected, lse_ctx = [], None
    for r in range(world):
        o, lse_ctx = cm.correct_attn_out(o_r[r].clone(), lse_r, r, None)
        corrected.append(o.float())
    o_ctx = torch.stack(corrected).sum(0).to(dtype)  # reduce_scatter sums in the model dtype
    out = torch.empty(T, H, D, dtype=dtype)
    out_lse = torch.empty(H, T, dtype=torch.float32)
    tm.merge_attn_states(out, o_ctx, lse_ctx.transpose(0, 1).contiguous(), s_out, s_lse, out_lse)
    f32 = lambda t: t.float().numpy()  # noqa: E731
    return dict(o_r=f32(o_r), lse_r=lse_r.numpy(), s_out=f32(s_out), s_lse=s_lse.numpy(),
                lse_ctx=lse_ctx.numpy(), o_ctx=f32(o_ctx), out=f32(out), out_lse=out_lse.numpy())


def main_dcp(meta):
    meta["dcp"] = {"slots": {}, "combine": {}}
    for name, (world, il, seed) in DCP_SLOT_CASES.items():
        np.savez_compressed(HERE / f"dcp_slots_{name}.npz", **dcp_slot_golden(world, il, seed))
        meta["dcp"]["slots"][name] = {"world": world, "interleave": il, "seed": seed}
        print(f"dcp_slots_{name}: written")
    for name, (world, dtype, seed) in DCP_COMBINE_CASES.items():
        np.savez_compressed(HERE / f"dcp_combine_{name}.npz", **dcp_combine_golden(world, dtype, seed))
        meta["dcp"]["combine"][name] = {"world": world, "dtype": str(dtype), "seed": seed}
        print(f"dcp_combine_{name}: written")


def main():
    only = sys.argv[sys.argv.index("--only") + 1] if "--only" in sys.argv else None
    if only in ("rope", "dcp"):
        meta = json.loads((HERE / "golden_meta.json").read_text())
        (main_rope if only == "rope" else main_dcp)(meta)
        (HERE / "golden_meta.json").write_text(json.dumps(meta, indent=1, default=str) + "\n")
        return
    attention_ref = load_attention_ref()
    meta = {"attention": {}, "append": {}}
    for name, spec in ATTN_CASES.items():
        arrays, cs = attention_golden(name, spec, attention_ref)
        np.savez_compressed(HERE / f"attn_{name}.npz", **arrays)
        meta["attention"][name] = {"spec": {k: v for k, v in spec.items()}, "input_checksum": cs}
        print(f"attn_{name}: out {arrays['out'].shape} checksum {cs:.6f}")
    from vllm.v1.attention.ops import triton_reshape_and_cache_flash as triton_mod

    for name, dtype, seed in (("bf16", torch.bfloat16, 21), ("fp32", torch.float32, 22)):
        arrays = append_golden(triton_mod, dtype, seed)
        np.savez_compressed(HERE / f"append_{name}.npz", **arrays)
        meta["append"][name] = {"dtype": str(dtype), "seed": seed}
        print(f"append_{name}: written")
    main_rope(meta)
    main_dcp(meta)
    (HERE / "golden_meta.json").write_text(json.dumps(meta, indent=1, default=str) + "\n")


if __name__ == "__main__":
    main()
