"""CPU oracle for the paged split-KV ("PS") attention path.

TEST INFRASTRUCTURE ONLY.  Nothing in the product imports this module; only
``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg use
it, and only as the checker.  It is a numpy restatement of the reference
semantics of vLLM 0.22's FlashAttention backend on sm_100 (the path prime-rl's
inference server runs):

* KV append  -- ``vllm/v1/attention/ops/triton_reshape_and_cache_flash.py:44-87``
  (NHD branch; the compiled ``reshape_and_cache_flash`` has the same contract,
  ``vllm/_custom_ops.py:2591-2610``).
* page gather through ``block_table`` -- the addressing FA4 uses for paged KV,
  ``vllm/vllm_flash_attn/cute/paged_kv.py:17-246``.
* attention  -- ``vllm/vllm_flash_attn/cute/testing.py:326-455`` (``attention_ref``:
  fp32 upcast, GQA head repeat, bottom-right causal mask, natural-log LSE).
* split-KV combine ("PS postprocess") --
  ``vllm/vllm_flash_attn/cute/flash_fwd_combine.py:521-567`` (LSE merge) and
  ``:633-640`` (weighted sum of partial outputs).
* split heuristic -- ``vllm/vllm_flash_attn/cute/interface.py:257-265``.

Parity pin: ``tests/golden/`` holds vectors produced by vLLM's own
``attention_ref`` (loaded by file path) and by vLLM's own Triton append kernel
run under the Triton CPU interpreter; ``tests/test_oracle.py`` checks this
module against them.
"""
from __future__ import annotations

import math

import numpy as np

LOG2E = math.log2(math.e)
LN2 = math.log(2.0)


# --------------------------------------------------------------------------
# KV append
# --------------------------------------------------------------------------
def kv_append(key, value, key_cache, value_cache, slot_mapping):
    """Scatter ``key``/``value`` rows into the paged cache in place.

    Follows ``triton_reshape_and_cache_flash.py:44-87`` (NHD layout):
    ``slot < 0`` is a padding token and is skipped (:46-48);
    ``block = slot // block_size``, ``offset = slot % block_size`` (:50-51);
    the whole ``[num_heads, head_size]`` row is copied (:78-87, :112-123).
    ``slot_mapping.shape[0]`` is the token count; key/value may be longer
    (``flash_attn.py:869-873``).

    key, value: [T', Hkv, D]; key_cache, value_cache: [NB, bs, Hkv, D].
    Works on any dtype because it is a byte copy.
    """
    slot_mapping = np.asarray(slot_mapping, dtype=np.int64)
    bs = key_cache.shape[1]
    for t, slot in enumerate(slot_mapping.tolist()):
        if slot < 0:
            continue
        blk, off = divmod(slot, bs)
        key_cache[blk, off] = key[t]
        value_cache[blk, off] = value[t]


def gather_pages(cache, block_table_row, seq_len):
    """Return the first ``seq_len`` token rows of one sequence: [L, Hkv, D].

    Page ``p`` of the sequence lives in cache block ``block_table_row[p]``;
    token ``i`` is row ``i % bs`` of page ``i // bs`` (``paged_kv.py:17-246``).
    """
    bs = cache.shape[1]
    npages = (seq_len + bs - 1) // bs
    if npages == 0:
        return cache[:0, 0]
    blocks = np.asarray(block_table_row[:npages], dtype=np.int64)
    rows = cache[blocks].reshape(npages * bs, *cache.shape[2:])
    return rows[:seq_len]


# --------------------------------------------------------------------------
# attention (attention_ref restated)
# --------------------------------------------------------------------------
def attention_ref(q, k, v, causal=True, softmax_scale=None):
    """Single-sequence attention, fp32, as ``testing.py:326-455``.

    q: [Sq, Hq, D]; k, v: [Sk, Hkv, D].  Returns (out [Sq, Hq, D] fp32,
    lse [Hq, Sq] fp32, natural log).

    * fp32 upcast (``upcast=True``, :352-354);
    * K/V heads repeated ``Hq // Hkv`` times, GQA group = consecutive q heads
      (:369-370);
    * ``scores = (q * scale) @ k^T`` (:375);
    * causal mask is bottom-right aligned: query row ``i`` may see key ``j``
      iff ``j <= i + Sk - Sq`` (``construct_local_mask`` :278-279 with
      ``window_size = (None, 0)``, :349-350);
    * ``lse = logsumexp(scores)`` (:428), ``out = softmax(scores) @ v`` (:430, :452);
    * a fully masked row gives ``out = 0`` (``attention.masked_fill`` at :438)
      and ``lse = -inf``.
    """
    q = np.asarray(q, dtype=np.float32)
    k = np.asarray(k, dtype=np.float32)
    v = np.asarray(v, dtype=np.float32)
    sq, hq, d = q.shape
    sk, hkv, _ = k.shape
    g = hq // hkv
    if softmax_scale is None:
        softmax_scale = 1.0 / math.sqrt(d)
    out = np.zeros((sq, hq, d), dtype=np.float32)
    lse = np.full((hq, sq), -np.inf, dtype=np.float32)
    if sk == 0 or sq == 0:
        return out, lse
    kk = np.repeat(k, g, axis=1)  # [Sk, Hq, D]
    vv = np.repeat(v, g, axis=1)
    # [Hq, Sq, Sk]
    scores = np.einsum("thd,shd->hts", q * np.float32(softmax_scale), kk, dtype=np.float32)
    if causal:
        row = np.arange(sq)[:, None]
        col = np.arange(sk)[None, :]
        masked = col > row + sk - sq
        scores = np.where(masked[None], np.float32(-np.inf), scores)
    mx = scores.max(axis=-1, keepdims=True)
    mx_safe = np.where(np.isfinite(mx), mx, np.float32(0.0))
    e = np.exp(scores - mx_safe, dtype=np.float32)
    ssum = e.sum(axis=-1, keepdims=True, dtype=np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        lse = (np.log(ssum) + mx_safe)[..., 0].astype(np.float32)
        p = np.where(ssum > 0, e / ssum, np.float32(0.0)).astype(np.float32)
    lse = np.where(ssum[..., 0] > 0, lse, np.float32(-np.inf))
    out = np.einsum("hts,shd->thd", p, vv, dtype=np.float32)
    return out.astype(np.float32), lse.astype(np.float32)


def paged_attention(q, key_cache, value_cache, block_table, seq_lens, query_start_loc,
                    softmax_scale, causal=True):
    """Varlen paged attention over a batch, the reference forward path.

    ``FlashAttentionImpl.forward`` (``flash_attn.py:787-817``) passes
    ``cu_seqlens_q = query_start_loc``, ``seqused_k = seq_lens`` and the
    block table to ``flash_attn_varlen_func``; sequence ``b`` owns query rows
    ``[qsl[b], qsl[b+1])`` and its first ``seq_lens[b]`` cached tokens.

    Returns (out [T, Hq, D] fp32, lse [Hq, T] fp32).
    """
    q = np.asarray(q, dtype=np.float32)
    t_total, hq, d = q.shape
    out = np.zeros((t_total, hq, d), dtype=np.float32)
    lse = np.full((hq, t_total), -np.inf, dtype=np.float32)
    qsl = np.asarray(query_start_loc, dtype=np.int64)
    for b, L in enumerate(np.asarray(seq_lens, dtype=np.int64).tolist()):
        t0, t1 = int(qsl[b]), int(qsl[b + 1])
        if t1 <= t0:
            continue
        kb = gather_pages(key_cache, block_table[b], L)
        vb = gather_pages(value_cache, block_table[b], L)
        o, l = attention_ref(q[t0:t1], kb, vb, causal=causal, softmax_scale=softmax_scale)
        out[t0:t1] = o
        lse[:, t0:t1] = l
    return out, lse


# --------------------------------------------------------------------------
# split-KV partials and the combine ("PS postprocess")
# --------------------------------------------------------------------------
def split_partials(q, k, v, splits, softmax_scale):
    """Per-split normalised partial outputs and LSEs of one decode query.

    q: [Hq, D] (the single decode token), k/v: [L, Hkv, D].  ``splits`` is a
    list of ``(start, end)`` key ranges.  An empty split has ``lse = -inf``
    and ``O = 0`` (``softmax.py:147-158`` zero-sum guard).
    Returns (o [S, Hq, D], lse [S, Hq]).
    """
    outs, lses = [], []
    for s0, s1 in splits:
        o, l = attention_ref(q[None], k[s0:s1], v[s0:s1], causal=False,
                             softmax_scale=softmax_scale)
        outs.append(o[0])
        lses.append(l[:, 0])
    return np.stack(outs).astype(np.float32), np.stack(lses).astype(np.float32)


def combine(o_partial, lse_partial):
    """Merge split partials, restating ``flash_fwd_combine.py``.

    o_partial: [S, ...rows, D] fp32 (normalised per split);
    lse_partial: [S, ...rows] fp32 natural-log LSE.

    * ``lse_max = max_s lse_s``; if every split is ``-inf`` the max used for
      the exponent is 0 (:541-547);
    * ``scale_s = exp2(lse_s*log2e - lse_max_cur*log2e)`` (:548-554);
    * ``lse = log(sum_s scale_s) + lse_max`` -- note: ``lse_max``, so an
      all-empty row yields ``-inf`` (:558);
    * ``inv_sum = 0`` when the sum is 0 or NaN, else ``1/sum`` (:560-562);
    * ``O = sum_s scale_s*inv_sum * O_s`` over splits with positive scale
      (:633-640).
    Returns (o [...rows, D], lse [...rows]).
    """
    o_partial = np.asarray(o_partial, dtype=np.float32)
    lse_partial = np.asarray(lse_partial, dtype=np.float32)
    lse_max = lse_partial.max(axis=0)
    lse_max_cur = np.where(lse_max == -np.inf, np.float32(0.0), lse_max)
    with np.errstate(over="ignore", invalid="ignore"):
        scale = np.exp2(lse_partial * np.float32(LOG2E) - lse_max_cur * np.float32(LOG2E),
                        dtype=np.float32)
    ssum = scale.sum(axis=0, dtype=np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        lse = (np.log(ssum) + lse_max).astype(np.float32)
        inv = np.where((ssum == 0) | np.isnan(ssum), np.float32(0.0), np.float32(1.0) / ssum)
    w = scale * inv
    w = np.where(w > 0, w, np.float32(0.0))
    o = (w[..., None] * o_partial).sum(axis=0, dtype=np.float32)
    return o.astype(np.float32), lse


def num_splits_heuristic(total_mblocks, num_sms, num_n_blocks, max_splits):
    """FA4's split count when ``num_splits < 1`` (``interface.py:257-265``)."""
    if num_n_blocks <= 4:
        return 1
    return min(num_sms // total_mblocks, max_splits, num_n_blocks)


# --------------------------------------------------------------------------
# seeded inputs for the benchmark configurations
# --------------------------------------------------------------------------
def decode_slots(block_table, seq_lens, block_size):
    """slot of the newest token of each sequence: ``bt[b, (L-1)//bs]*bs + (L-1)%bs``."""
    bt = np.asarray(block_table, dtype=np.int64)
    L = np.asarray(seq_lens, dtype=np.int64)
    pos = L - 1
    return bt[np.arange(len(L)), pos // block_size] * block_size + pos % block_size


# --------------------------------------------------------------------------
# Shared-prefix (cascade) plan and cascade attention
# --------------------------------------------------------------------------
def cascade_plan(block_table, seq_lens, query_start_loc=None, block_size=16,
                 min_shared_pages=8, enabled=True):
    """Groups of adjacent decode sequences with identical leading pages.

    The batch-wide rule vLLM applies (``flash_attn.py:1088-1130``,
    ``use_cascade_attention``: one prefix common to every request) made per
    group, read off the block table the way prefix caching lays it out
    (shared prompt blocks have one physical id):

    * ``full(b) = (seq_len - 1) // 16`` complete 16-token pages before the page
      of the last token (0 unless sequence b has exactly one query row);
    * ``shared(b)``: leading pages whose block entries equal row ``b-1``'s,
      capped at ``min(full(b), full(b-1))``; ``shared(0) = 0``;
    * ``b`` starts a group if ``b == 0``, ``shared(b) < min_shared_pages`` or
      ``shared(b) < shared(b+1)``;
    * a group's pages = min of ``shared`` over its members after the first;
      groups of >= 2 members are listed in order.

    Returns a dict with the plan's arrays (int lists).
    """
    bt = np.asarray(block_table)
    L = np.asarray(seq_lens, dtype=np.int64)
    B = len(L)
    sub = block_size // 16
    maxp = bt.shape[1] * sub if bt.ndim == 2 else 0
    qlen = (np.diff(np.asarray(query_start_loc, dtype=np.int64)) if query_start_loc is not None
            else np.ones(B, dtype=np.int64))

    def full(b):
        if qlen[b] != 1 or L[b] < 1:
            return 0
        return int(min((L[b] - 1) // 16, maxp))

    shared = [0] * B
    if enabled:
        for b in range(1, B):
            F = min(full(b), full(b - 1))
            E = (F + sub - 1) // sub
            m = 0
            while m < E and bt[b, m] == bt[b - 1, m]:
                m += 1
            shared[b] = min(m * sub, F)

    def starts(b):
        return b == 0 or shared[b] < min_shared_pages or (b + 1 < B and shared[b] < shared[b + 1])

    groups = []  # [first, size, pages]
    for b in range(B):
        if starts(b):
            groups.append([b, 1, None])
        else:
            grp = groups[-1]
            grp[1] += 1
            grp[2] = shared[b] if grp[2] is None else min(grp[2], shared[b])
    seq_group = [-1] * B
    listed = []
    for first, size, pages in groups:
        if size >= 2:
            for b in range(first, first + size):
                seq_group[b] = len(listed)
            listed.append((first, size, pages))
    return {
        "num_groups": len(listed),
        "seq_group": seq_group,
        "group_first": [g[0] for g in listed],
        "group_size": [g[1] for g in listed],
        "group_pages": [g[2] for g in listed],
        "shared_pages": shared,
    }


def cascade_decode(q, key_cache, value_cache, block_table, seq_lens, plan, softmax_scale):
    """Decode attention evaluated the cascade way, for one query row per sequence.

    For a grouped sequence: attention over the group's shared pages (read
    from the first member's table) and over its own remaining pages, merged
    with :func:`combine` -- what ``cascade_attention`` + ``merge_attn_states``
    compute (``flash_attn.py:1132-1223``).  It equals
    :func:`paged_attention` up to fp32 rounding; the tests use it to show the
    prefix/suffix split is exact.
    """
    q = np.asarray(q, dtype=np.float32)
    B = len(seq_lens)
    Hq = q.shape[1]
    out = np.zeros_like(q)
    lse = np.full((Hq, B), -np.inf, dtype=np.float32)
    for b in range(B):
        Lb = int(seq_lens[b])
        k = gather_pages(key_cache, block_table[b], Lb)
        v = gather_pages(value_cache, block_table[b], Lb)
        g = plan["seq_group"][b]
        cut = 16 * plan["group_pages"][g] if g >= 0 else 0
        parts = [(0, cut), (cut, Lb)] if cut > 0 else [(0, Lb)]
        os_, ls_ = [], []
        for lo, hi in parts:
            o, l = attention_ref(q[b:b + 1], k[lo:hi], v[lo:hi], causal=False,
                                 softmax_scale=softmax_scale)
            os_.append(o[0])
            ls_.append(l[:, 0])
        o, l = combine(np.stack(os_), np.stack(ls_))
        out[b] = o
        lse[:, b] = l
    return out, lse


# --------------------------------------------------------------------------
# Rotary embedding (fused RoPE + KV append)
# --------------------------------------------------------------------------
def round_to(x, dtype):
    """Round float32 values to ``dtype`` ("bf16", "fp16" or "fp32") and back,
    round-to-nearest-even (what torch does after every bf16/fp16 operation)."""
    x = np.asarray(x, dtype=np.float32)
    if dtype == "fp32":
        return x
    if dtype == "fp16":
        return x.astype(np.float16).astype(np.float32)
    bits = x.view(np.uint32).astype(np.uint64)
    nan = np.isnan(x)
    rounded = ((bits + 0x7FFF + ((bits >> 16) & 1)) >> 16) << 16
    out = (rounded & 0xFFFFFFFF).astype(np.uint32).view(np.float32)
    return np.where(nan, x, out).astype(np.float32)


def rope(x, positions, cos_sin_rows, rotary_dim, is_neox, dtype):
    """Rotary embedding of ``x`` [T, H, D] (float32 holding ``dtype`` values).

    Restates ``RotaryEmbedding.forward_static`` /
    ``ApplyRotaryEmb.forward_static``
    (``vllm/model_executor/layers/rotary_embedding/base.py:140-181``,
    ``common.py:144-180``): ``cos, sin = cos_sin_cache[positions].chunk(2)``
    cast to the model dtype; neox style pairs element ``i`` with ``i + rot/2``,
    GPT-J style ``2i`` with ``2i + 1``; ``o1 = x1*cos - x2*sin``, ``o2 =
    x2*cos + x1*sin`` with every product and sum rounded to the model dtype
    (torch's bf16/fp16 tensor arithmetic); dims past ``rotary_dim`` pass
    through.  ``cos_sin_rows`` [T, rot] are the cache rows at ``positions``.
    """
    x = np.asarray(x, dtype=np.float32)
    out = x.copy()
    half = rotary_dim // 2
    cs = round_to(np.asarray(cos_sin_rows, dtype=np.float32), dtype)
    cos = cs[:, None, :half]
    sin = cs[:, None, half:rotary_dim]
    if is_neox:
        x1, x2 = x[..., :half], x[..., half:rotary_dim]
    else:
        x1, x2 = x[..., 0:rotary_dim:2], x[..., 1:rotary_dim:2]
    o1 = round_to(round_to(x1 * cos, dtype) - round_to(x2 * sin, dtype), dtype)
    o2 = round_to(round_to(x2 * cos, dtype) + round_to(x1 * sin, dtype), dtype)
    if is_neox:
        out[..., :half], out[..., half:rotary_dim] = o1, o2
    else:
        out[..., 0:rotary_dim:2], out[..., 1:rotary_dim:2] = o1, o2
    return out


# --------------------------------------------------------------------------
# decode context parallelism (DCP)
# --------------------------------------------------------------------------
def dcp_local_lens(lens, world, rank, interleave=1):
    """Tokens of each length-``lens`` prefix stored by ``rank``: positions p
    with ``(p // interleave) % world == rank``.  Restates
    ``get_dcp_local_seq_lens`` (``vllm/v1/attention/backends/utils.py:857-894``):
    ``base = L // I // N * I``, ``rem = L - base * N``,
    ``local = base + clip(rem - rank * I, 0, I)``."""
    L = np.asarray(lens, dtype=np.int64)
    base = L // interleave // world * interleave
    rem = L - base * world
    return (base + np.clip(rem - rank * interleave, 0, interleave)).astype(np.int32)


def dcp_placement(positions, block_table_row, block_size, world, rank, interleave=1):
    """Local slot of each position on ``rank`` (-1 where another rank stores
    it), restating ``_compute_slot_mapping_kernel``
    (``vllm/v1/worker/block_table.py:326-380``): virtual blocks of
    ``block_size * world`` positions; offset ``o`` of a virtual block is
    stored by rank ``(o // I) % world`` at ``(o // (world*I)) * I + o % I`` of
    the block ``block_table_row[pos // (block_size*world)]``."""
    pos = np.asarray(positions, dtype=np.int64)
    vbs = block_size * world
    blk = pos // vbs
    o = pos - blk * vbs
    local = (o // interleave) % world == rank
    off = (o // (world * interleave)) * interleave + o % interleave
    slots = np.asarray(block_table_row, dtype=np.int64)[blk] * block_size + off
    return np.where(local, slots, -1)


def dcp_decode(q_all, key_caches, value_caches, block_table, seq_lens, new_key, new_value,
               softmax_scale, interleave=1, partial_dtype="fp32"):
    """One DCP decode step of the whole group, the way vLLM evaluates it
    (``FlashAttentionImpl._forward_with_dcp``, ``flash_attn.py:885-983``):

    * rank r attends with every query head over its context slice (the first
      ``dcp_local_lens(seq_lens - 1, ...)`` local tokens, non-causal), giving
      ``(o_r, lse_r)``; ``o_r`` is stored in ``partial_dtype`` (vLLM: the model
      dtype);
    * ``correct_attn_out`` (``ops/common.py:42-96``): NaN and +inf LSEs count
      as -inf, ``lse = log(sum_r exp(lse_r - m)) + m`` with a max of -inf
      counted as 0, ``o_r *= exp(lse_r - lse)`` (NaN/+inf exponents -> 0);
      the reduce_scatter sums the corrected ``o_r`` over ranks;
    * the new token attends to itself (``o = v``, ``lse = scale * q.k``) and
      ``merge_attn_states`` (``triton_merge_attn_states.py:58-140``) merges it.

    q_all [T, Hq, D]; key_caches/value_caches: per rank [NB, bs, Hkv, D];
    new_key/new_value [T, Hkv, D].  Returns (out [T, Hq, D], lse [Hq, T]) fp32
    for all heads (rank r keeps heads [r*Hq/N, (r+1)*Hq/N)).
    """
    q_all = np.asarray(q_all, dtype=np.float32)
    T, hq, d = q_all.shape
    world = len(key_caches)
    ctx = np.asarray(seq_lens, dtype=np.int64) - 1
    qsl = np.arange(T + 1)
    outs, lses = [], []
    for r in range(world):
        lens_r = dcp_local_lens(ctx, world, r, interleave)
        o, l = paged_attention(q_all, key_caches[r], value_caches[r], block_table, lens_r, qsl,
                               softmax_scale, causal=False)
        outs.append(round_to(o, partial_dtype))
        lses.append(l)
    k = np.asarray(new_key, dtype=np.float32)
    v = np.asarray(new_value, dtype=np.float32)
    g = hq // k.shape[1]
    kk, vv = np.repeat(k, g, axis=1), np.repeat(v, g, axis=1)
    s_lse = (np.float32(softmax_scale) * np.einsum("thd,thd->ht", q_all, kk)).astype(np.float32)
    out, lse, _, _ = dcp_combine(np.stack(outs), np.stack(lses), vv, s_lse)
    return out, lse


def dcp_combine(o_r, lse_r, s_out, s_lse, rounding="fp32"):
    """The cross-rank half of a DCP decode step.

    o_r [N, T, H, D], lse_r [N, H, T]: every rank's partial output and LSE;
    s_out [T, H, D], s_lse [H, T]: the new tokens' attention over themselves.
    ``correct_attn_out`` (``ops/common.py:42-96``) then the sum over ranks
    (``reduce_scatter``, ``common.py:218``) then ``merge_attn_states``
    (``triton_merge_attn_states.py:58-140``).  ``rounding`` = "bf16"/"fp16"
    rounds where vLLM stores in the model dtype (each corrected partial, their
    sum, the merged output); "fp32" rounds nowhere.
    Returns (out [T, H, D], lse [H, T], o_ctx [T, H, D], lse_ctx [H, T]).
    """
    o_r = np.asarray(o_r, dtype=np.float32)
    lse_r = np.asarray(lse_r, dtype=np.float32)
    lse_r = np.where(np.isnan(lse_r) | (lse_r == np.inf), -np.inf, lse_r).astype(np.float32)
    m = lse_r.max(axis=0)
    m = np.where(m == -np.inf, 0.0, m).astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        lse_ctx = (np.log(np.exp(lse_r - m).sum(axis=0)) + m).astype(np.float32)
        f = lse_r - lse_ctx
    f = np.where(np.isnan(f) | (f == np.inf), -np.inf, f)
    fac = np.exp(f).astype(np.float32)  # [N, H, T]
    corrected = round_to(o_r * np.transpose(fac, (0, 2, 1))[..., None], rounding)
    o_ctx = round_to(corrected.sum(axis=0), rounding)
    out, lse = merge_states(o_ctx, lse_ctx, s_out, s_lse)
    return round_to(out, rounding), lse, o_ctx, lse_ctx.astype(np.float32)


def merge_states(p_out, p_lse, s_out, s_lse):
    """``merge_attn_states`` (``triton_merge_attn_states.py:58-140``): two
    partial attentions over disjoint key sets, outputs [T, H, D] and LSEs
    [H, T]; +inf LSEs count as -inf.  Returns (out, lse)."""
    p_out = np.asarray(p_out, dtype=np.float32)
    s_out = np.asarray(s_out, dtype=np.float32)
    p = np.asarray(p_lse, dtype=np.float32)
    s = np.asarray(s_lse, dtype=np.float32)
    p = np.where(p == np.inf, -np.inf, p)
    s = np.where(s == np.inf, -np.inf, s)
    mx = np.maximum(p, s)
    with np.errstate(invalid="ignore"):
        pse, sse = np.exp(p - mx), np.exp(s - mx)
    tot = pse + sse
    out = p_out * (pse / tot).T[..., None] + s_out * (sse / tot).T[..., None]
    return out.astype(np.float32), (np.log(tot) + mx).astype(np.float32)


def dcp_prefill(q_all, key_caches, value_caches, block_table, seq_lens, query_start_loc, new_key,
                new_value, softmax_scale, interleave=1):
    """A DCP step with multi-token query chunks, the way vLLM evaluates it
    (``FlashAttentionImpl._forward_with_dcp``, ``flash_attn.py:885-983``):

    * the context of sequence b is its first ``seq_lens[b] - q_len(b)``
      tokens; rank r attends from every query row over its slice of them,
      non-causally (all of the context precedes the chunk);
    * the ranks' partials are corrected and summed (``cp_lse_ag_out_rs``);
    * the chunk attends causally over its own new keys/values
      (``flash_attn_varlen_func(q, key, value, cu_seqlens_q, cu_seqlens_k =
      cu_seqlens_q, causal=True)``);
    * ``merge_attn_states`` merges the two.

    q_all [T, Hq, D] (rows in ``query_start_loc`` order); key_caches /
    value_caches: per rank [NB, bs, Hkv, D] holding the context only;
    new_key / new_value [T, Hkv, D].  Returns (out [T, Hq, D], lse [Hq, T]).
    """
    q_all = np.asarray(q_all, dtype=np.float32)
    T, hq, d = q_all.shape
    world = len(key_caches)
    qsl = np.asarray(query_start_loc, dtype=np.int64)
    L = np.asarray(seq_lens, dtype=np.int64)
    ctx = L - np.diff(qsl)
    outs, lses = [], []
    for r in range(world):
        lens_r = dcp_local_lens(ctx, world, r, interleave)
        o, l = paged_attention(q_all, key_caches[r], value_caches[r], block_table, lens_r, qsl,
                               softmax_scale, causal=False)
        outs.append(o)
        lses.append(l)
    _, _, o_ctx, lse_ctx = dcp_combine(np.stack(outs), np.stack(lses), np.zeros_like(q_all),
                                       np.full((hq, T), -np.inf, np.float32))
    o_q = np.zeros_like(q_all)
    lse_q = np.full((hq, T), -np.inf, np.float32)
    k = np.asarray(new_key, dtype=np.float32)
    v = np.asarray(new_value, dtype=np.float32)
    for b in range(len(L)):
        t0, t1 = int(qsl[b]), int(qsl[b + 1])
        if t1 > t0:
            o, l = attention_ref(q_all[t0:t1], k[t0:t1], v[t0:t1], causal=True,
                                 softmax_scale=softmax_scale)
            o_q[t0:t1], lse_q[:, t0:t1] = o, l
    return merge_states(o_ctx, lse_ctx, o_q, lse_q)


# --------------------------------------------------------------------------
# fp8 (e4m3) KV cache
# --------------------------------------------------------------------------
def _e4m3_values():
    """Value of each non-negative e4m3fn code 0..126 (0x7F is NaN): 4
    exponent bits with bias 7, 3 mantissa bits, subnormals at exponent 0,
    no infinities (OCP 8-bit floating point, E4M3)."""
    codes = np.arange(127)
    e, m = codes >> 3, codes & 7
    return np.where(e == 0, m / 8.0 * 2.0 ** -6, (1 + m / 8.0) * 2.0 ** (e - 7.0))


_E4M3 = _e4m3_values()


def e4m3_encode(x):
    """float32 -> e4m3fn codes (uint8): nearest value, ties to the even
    code, magnitudes past 448 saturate to 448 (the ``satfinite`` conversion
    of CUDA's ``__nv_cvt_float_to_fp8`` and of Triton's fp8 store), NaN ->
    0x7F."""
    x = np.asarray(x, dtype=np.float32)
    a = np.abs(x).astype(np.float64)
    hi = np.clip(np.searchsorted(_E4M3, a), 0, 126)
    lo = np.clip(hi - 1, 0, 126)
    dlo, dhi = np.abs(a - _E4M3[lo]), np.abs(_E4M3[hi] - a)
    pick = np.where(dlo < dhi, lo, np.where(dhi < dlo, hi, np.where(lo % 2 == 0, lo, hi)))
    pick = np.where(a >= 448.0, 126, pick)
    code = pick.astype(np.uint8) | (np.signbit(x).astype(np.uint8) << 7)
    return np.where(np.isnan(x), np.uint8(0x7F), code).astype(np.uint8)


def e4m3_decode(codes):
    """e4m3fn codes (uint8) -> float32."""
    c = np.asarray(codes, dtype=np.uint8)
    mag = c & 0x7F
    v = np.where(mag == 0x7F, np.nan, _E4M3[np.minimum(mag, 126)])
    return np.where(c & 0x80, -v, v).astype(np.float32)


def kv_append_fp8(key, value, key_cache, value_cache, slot_mapping, k_scale, v_scale):
    """``reshape_and_cache_flash`` with kv_cache_dtype "fp8"
    (``triton_reshape_and_cache_flash.py:93-110``): rows stored as
    e4m3(x / k_scale) and e4m3(x / v_scale), the quotient in float32.
    Caches are uint8 code arrays, updated in place."""
    ks, vs = np.float32(k_scale), np.float32(v_scale)
    kq = e4m3_encode(np.asarray(key, dtype=np.float32) / ks)
    vq = e4m3_encode(np.asarray(value, dtype=np.float32) / vs)
    kv_append(kq, vq, key_cache, value_cache, slot_mapping)


def dequantize_cache(codes, scale):
    """An fp8 cache read as attention sees it: code * scale, float32."""
    return (e4m3_decode(codes) * np.float32(scale)).astype(np.float32)
