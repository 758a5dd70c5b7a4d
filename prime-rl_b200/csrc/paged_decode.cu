// Paged split-KV decode attention for sm_100a, with the split combine fused.
//
// Semantics: vllm/vllm_flash_attn/cute/testing.py:326-455 (attention_ref: fp32
// softmax(q k^T * scale) v, GQA head groups, natural-log LSE) evaluated over the
// paged cache the way FA4 reads it (cute/paged_kv.py), with FA4's split-KV
// combine (cute/flash_fwd_combine.py:521-567 LSE merge, :633-640 weighted sum)
// and FA4's zero-sum guard (cute/softmax.py:147-158).
//
// Work decomposition ("stream-K" over page-heads):
//   A unit of work is one 16-token page of one KV head of one sequence (two
//   consecutive pages with an fp8 cache).  The units ("page-heads") of the
//   batch are laid out in (sequence, kv head, page) order and cut into equal
//   contiguous ranges, one per warp of a persistent grid of one CTA per SM.  A warp therefore streams an exactly equal share of the KV
//   bytes.  Where a warp's range crosses a (sequence, kv head) boundary it
//   finishes that segment as a split: it writes a normalised fp32 partial and
//   its LSE, bumps a per-(sequence, kv head) counter, and the warp that brings
//   the counter to the split count merges all partials (no waiting, so no
//   spin).  A segment that fits in one warp's range writes the output directly.
//
// Shared-prefix ("cascade") mode: with a plan of groups of adjacent sequences
//   whose leading block-table entries are identical (GRPO samples of one
//   prompt), the page-head list starts with prefix segments: (group, kv head,
//   pass) streams the group's shared pages once for up to 16 query columns
//   (members x GQA heads) instead of once per member.  Each member's own
//   segment starts after the prefix.  The prefix result enters every member's
//   combine as one more split, so the output is the same softmax over the same
//   keys (vLLM's cascade_attention + merge_attn_states,
//   vllm/v1/attention/backends/flash_attn.py:1132-1223, generalised from one
//   batch-wide prefix to per-group prefixes).
//
// Per warp: a private ring of kDecodeStages page buffers in shared memory, each
// filled by four TMA tensor loads (K lo/hi 64 dims, V lo/hi) of a 16-token
// page, 128-byte swizzled, completion on an mbarrier.  The first page of a
// segment also carries the segment's GQA query rows (cp.async.bulk, one
// 256-byte row per head) into a padded per-warp slot, so a segment start costs
// no dependent global load.  Block-table entries are fetched 32 at a time into
// a warp register and handed out by shuffle.
//
// Compute per page, with tokens on the MMA M axis and the GQA group on N
// (m16n8k16):
//   S^T[16 tok, 8 heads]   = K[16 tok, 128] . Q^T          (8 mma, K via ldmatrix)
//   online softmax per head column (exp2 domain; 3 xor-shuffles per max)
//   P^T -> B fragment      via movmatrix.trans (no shared-memory round trip)
//   O^T[128 dims, 8 heads] += V^T[128, 16 tok] . P^T        (8 mma, V via ldmatrix.trans)
//
// Fused head all-gather (KV-head-sharded groups, DecodeParams::gather_world):
//   every output row is also stored into each peer GPU's slab over NVLink as
//   it is finished -- by the combine (one 256-byte row per warp store) or, for
//   a segment one warp streamed alone, from the accumulators transposed by
//   movmatrix -- so the exchange overlaps the streaming of the remaining pages.  At the end
//   each CTA waits (bounded) for every rank's "rows written" flag and copies
//   the peers' rows from this GPU's slab into the output; a second flag round
//   ("rows copied") keeps the next call from overwriting rows a peer has not
//   copied yet.
#include "peer_sync.cuh"
#include "ps_common.cuh"
#include "ps_launch.h"

namespace ps {

constexpr int kPageTokens = 16;
constexpr int kHeadDim = 128;
constexpr int kBoxBytes = kPageTokens * 64 * 2;  // 2 KB: 16 rows x 128 bytes
constexpr int kStageBytes = 4 * kBoxBytes;       // K lo, K hi, V lo, V hi
// fp8 (e4m3) cache: one box per page of K or V, 16 rows x 128 one-byte dims
constexpr int kBoxBytesF8 = kPageTokens * kHeadDim;  // 2 KB
constexpr int kQRowBytes = kHeadDim * 2 + 16;    // padded query row (conflict-free ldmatrix)
constexpr int kPrefixNT = 2;                     // prefix segments: 16 query columns
#ifndef PS_CASCADE_PREFIX_COST16
#define PS_CASCADE_PREFIX_COST16 26
#endif
// Streaming time of a prefix page-head (16 query columns) relative to an own
// page-head, in sixteenths: the stream-K cut weights the two kinds by it.
constexpr int kCascadePrefixCost16 = PS_CASCADE_PREFIX_COST16;

enum { kPlain = 0, kCasPrefix = 1, kCasSuffix = 2 };

// Split-slot record: kRec output rows of 128 fp32, then kRec fp32 LSEs.
template <int kRec>
__device__ __forceinline__ float* slot_o(const DecodeParams& p, int64_t slot, int row) {
  return p.part + slot * (kRec * (kHeadDim + 1)) + row * kHeadDim;
}
template <int kRec>
__device__ __forceinline__ float* slot_lse(const DecodeParams& p, int64_t slot, int row) {
  return p.part + slot * (kRec * (kHeadDim + 1)) + kRec * kHeadDim + row;
}

// Shared-memory tables built by the prologue.
struct Tables {
  const int* prefix;  // [B+1] exclusive scan of each sequence's own units (pages; fp8: page pairs)
  const int* soff;    // [B]   cascade: pages of the sequence covered by its group prefix
  const int* gph;     // [G+1] cascade: exclusive scan of pages * passes per group
  const int* gu;      // [G+1] cascade: exclusive scan of passes per group
  int G;
  int mpp;            // cascade: group members per 16-column pass
  int64_t pre_total;  // page-heads in the prefix region (Hkv * gph[G])
  int64_t pre_units;  // prefix segments (Hkv * gu[G])
  // Cost-weighted partition: a prefix page-head costs wp, an own one wo, and
  // warp w streams the list positions whose cost offset lies in [w*Qc,
  // (w+1)*Qc).  Qc >= max(wp, wo), so the non-empty ranges are exactly those
  // of the first warps: a segment's split count is the number of warps its
  // pages span.
  int wp, wo;
  int64_t Qc;
};

// Cost offset of list position i, and the warp that streams it.
__device__ __forceinline__ int64_t list_cost(const Tables& tb, int64_t i) {
  return i < tb.pre_total ? i * tb.wp : tb.pre_total * tb.wp + (i - tb.pre_total) * tb.wo;
}
__device__ __forceinline__ int64_t warp_of(const Tables& tb, int64_t i) {
  return list_cost(tb, i) / tb.Qc;
}
// First list position whose cost offset is >= X.
__device__ __forceinline__ int64_t list_at_cost(const Tables& tb, int64_t X) {
  const int64_t xp = tb.pre_total * tb.wp;
  if (X <= xp) return (X + tb.wp - 1) / tb.wp;
  return tb.pre_total + (X - xp + tb.wo - 1) / tb.wo;
}

// Position in the page-head list.  Own segments: (b, h, page p of P, first page
// `off`).  Prefix segments: b = first member, g = group, pass of `passes`,
// `ncols` query columns, P = shared pages.
struct Cursor {
  int b, h, p, P, off;
  int g, pass, passes, ncols;
};

__device__ __forceinline__ int seq_pages(const int* prefix, int b) {
  return prefix[b + 1] - prefix[b];
}

template <int kMode>
__device__ __forceinline__ void load_group(Cursor& c, const DecodeParams& p, const Tables& tb) {
  c.b = __ldg(p.cas_group_first + c.g);
  const int size = __ldg(p.cas_group_size + c.g);
  c.P = __ldg(p.cas_group_pages + c.g);
  c.passes = (size + tb.mpp - 1) / tb.mpp;
  c.ncols = min(tb.mpp, size - c.pass * tb.mpp) * p.group;
}

// Advance to the next page-head in list order.
template <int kMode>
__device__ __forceinline__ void cursor_next(Cursor& c, const DecodeParams& p, const Tables& tb,
                                            int num_kv_heads) {
  if (++c.p < c.P) return;
  c.p = 0;
  if constexpr (kMode == kCasPrefix) {
    if (++c.pass < c.passes) {
      const int size = __ldg(p.cas_group_size + c.g);
      c.ncols = min(tb.mpp, size - c.pass * tb.mpp) * p.group;
      return;
    }
    c.pass = 0;
    if (++c.h < num_kv_heads) {
      c.ncols = min(tb.mpp, __ldg(p.cas_group_size + c.g)) * p.group;
      return;
    }
    c.h = 0;
    ++c.g;  // the caller never advances past the region's last page-head
    load_group<kMode>(c, p, tb);
  } else {
    if (++c.h < num_kv_heads) return;
    c.h = 0;
    do {
      ++c.b;
      c.P = seq_pages(tb.prefix, c.b);
    } while (c.P == 0);
    if constexpr (kMode == kCasSuffix) c.off = tb.soff[c.b];
  }
}

// Locate page-head gi of the region; requires gi < the region's size.
template <int kMode>
__device__ __forceinline__ Cursor cursor_at(int64_t gi, const DecodeParams& p, const Tables& tb,
                                            int num_kv_heads) {
  Cursor c;
  c.off = 0;
  c.g = c.pass = c.passes = c.ncols = 0;
  if constexpr (kMode == kCasPrefix) {
    int lo = 0, hi = tb.G - 1;  // largest g with gph[g]*Hkv <= gi
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (static_cast<int64_t>(tb.gph[mid]) * num_kv_heads <= gi)
        lo = mid;
      else
        hi = mid - 1;
    }
    c.g = lo;
    c.pass = 0;
    load_group<kMode>(c, p, tb);
    const int64_t r = gi - static_cast<int64_t>(tb.gph[lo]) * num_kv_heads;
    const int64_t per = static_cast<int64_t>(c.passes) * c.P;
    c.h = static_cast<int>(r / per);
    const int64_t rem = r - static_cast<int64_t>(c.h) * per;
    c.pass = static_cast<int>(rem / c.P);
    c.p = static_cast<int>(rem - static_cast<int64_t>(c.pass) * c.P);
    const int size = __ldg(p.cas_group_size + c.g);
    c.ncols = min(tb.mpp, size - c.pass * tb.mpp) * p.group;
  } else {
    int lo = 0, hi = p.num_seqs - 1;  // largest b with prefix[b]*Hkv <= gi
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (static_cast<int64_t>(tb.prefix[mid]) * num_kv_heads <= gi)
        lo = mid;
      else
        hi = mid - 1;
    }
    c.b = lo;
    c.P = seq_pages(tb.prefix, lo);
    const int64_t r = gi - static_cast<int64_t>(tb.prefix[lo]) * num_kv_heads;
    c.h = static_cast<int>(r / c.P);
    c.p = static_cast<int>(r - static_cast<int64_t>(c.h) * c.P);
    if constexpr (kMode == kCasSuffix) c.off = tb.soff[lo];
  }
  return c;
}

template <bool kBF16>
__device__ __forceinline__ void store_out2(void* out, int64_t idx, float v) {
  if constexpr (kBF16)
    reinterpret_cast<__nv_bfloat16*>(out)[idx] = __float2bfloat16_rn(v);
  else
    reinterpret_cast<__half*>(out)[idx] = __float2half_rn(v);
}

__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(gsrc)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void fence_acq_rel_gpu() {
  asm volatile("fence.acq_rel.gpu;" ::: "memory");
}

// Atomic add with release semantics at gpu scope: the caller's earlier writes
// (and, cumulatively, its warp's, ordered by __syncwarp) are visible before
// the new count is.
__device__ __forceinline__ int atomic_add_release_gpu(int* addr, int v) {
  int old;
  asm volatile("atom.add.release.gpu.global.s32 %0, [%1], %2;" : "=r"(old) : "l"(addr), "r"(v) : "memory");
  return old;
}

// Merge partial records.  Sources: slots [slot0, slot0 + n) rows [0, nrows)
// and, when xslot >= 0, slot xslot rows [xrow0, xrow0 + nrows).  FA4 combine:
// lse_max over sources (0 if all -inf), scale_s = exp2((lse_s - lse_max_cur) *
// log2e), lse = log(sum) + lse_max, inv = 0 for a zero/NaN sum, O = sum_s
// scale_s * inv * O_s over sources with scale > 0.
// kToRecord: row j goes to record dst_slot row j (fp32; dst_slot may be slot0:
// every read of a row precedes its write), else to out/lse of sequence b,
// query heads h * group + j.
template <bool kBF16, int kRec, bool kToRecord>
__device__ __noinline__ void combine_rows(const DecodeParams& p, int64_t slot0, int n,
                                          int64_t xslot, int xrow0, int nrows, int b, int h,
                                          int64_t dst_slot, int lane) {
  const int group = p.group;
  const int ntot = n + (xslot >= 0 ? 1 : 0);
  const int qrow = kToRecord ? 0 : (p.qsl ? __ldg(p.qsl + b) : b);
  const float kLog2e = 1.4426950408889634f;
  auto src_slot = [&](int k) { return k < n ? slot0 + k : xslot; };
  auto src_row = [&](int k, int j) { return k < n ? j : xrow0 + j; };
  auto emit = [&](int j, float4 acc, float lse) {
    if constexpr (kToRecord) {
      reinterpret_cast<float4*>(slot_o<kRec>(p, dst_slot, j))[lane] = acc;
      if (lane == 0) *slot_lse<kRec>(p, dst_slot, j) = lse;
    } else {
      const int qh = h * group + j;
      const int64_t obase = qrow * p.o_st + qh * p.o_sh + lane * 4;
      uint2 packed;
      packed.x = pack2<kBF16>(acc.x, acc.y);
      packed.y = pack2<kBF16>(acc.z, acc.w);
      if constexpr (kBF16)
        *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(p.out) + obase) = packed;
      else
        *reinterpret_cast<uint2*>(reinterpret_cast<__half*>(p.out) + obase) = packed;
      if (lane == 0 && p.lse != nullptr) p.lse[qh * p.lse_sh + qrow * p.lse_st] = lse;
      if (p.gather_world > 0) {
        // the same row into every peer's slab (the warp's 8-byte lane stores
        // form one 256-byte row); a row past the slabs' tokens is refused
        if (qrow < p.gather_tokens) {
#pragma unroll
          for (int r = 0; r < 8; ++r) {
            char* dst = r < p.gather_world ? p.gather_rows[r] : nullptr;
            if (dst != nullptr)
              *reinterpret_cast<uint2*>(dst + qrow * p.gather_row_st + qh * 256 + lane * 8) = packed;
          }
        } else if (lane == 0) {
          set_status(p.gather_status, PS_DEV_BAD_METADATA);
        }
      }
    }
  };
  if (kRec == 8 && ntot <= 4 && nrows <= 4) {
    // few sources (the common split count): every partial row this lane
    // needs is loaded together with the LSEs, so the merge waits on one L2
    // round trip instead of two (8-column kernels only: the 16-column ones
    // have no registers to spare for it)
    float4 ov[4][4];
    float ls[4][4];
#pragma unroll
    for (int k = 0; k < 4; ++k)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const bool use = k < ntot && j < nrows;
        ov[k][j] = use ? __ldcg(reinterpret_cast<const float4*>(slot_o<kRec>(p, src_slot(k), src_row(k, j))) + lane)
                       : make_float4(0.f, 0.f, 0.f, 0.f);
        ls[k][j] = use ? __ldcg(slot_lse<kRec>(p, src_slot(k), src_row(k, j))) : -INFINITY;
      }
    __syncwarp();  // every lane's reads precede the writes
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (j >= nrows) break;
      const float mx = fmaxf(fmaxf(ls[0][j], ls[1][j]), fmaxf(ls[2][j], ls[3][j]));
      const float mx_cur = (mx == -INFINITY) ? 0.f : mx;
      float e[4], sum = 0.f;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        e[k] = k < ntot ? ex2(ls[k][j] * kLog2e - mx_cur * kLog2e) : 0.f;
        sum += e[k];
      }
      const float inv = (sum == 0.f || sum != sum) ? 0.f : 1.f / sum;
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float w = e[k] * inv;
        acc.x += w * ov[k][j].x;
        acc.y += w * ov[k][j].y;
        acc.z += w * ov[k][j].z;
        acc.w += w * ov[k][j].w;
      }
      emit(j, acc, __logf(sum) + mx);
    }
    return;
  }
  if (ntot <= 32) {
    // fast path: lane k owns source k; one LSE load per lane and row, and the
    // O loads of a phase are independent of one another and of the weights
    // (an empty source has weight 0 and an all-zero partial, so every source
    // is accumulated unconditionally).  Rows in chunks of 4 keep the register
    // footprint small.
    const int64_t my_slot = src_slot(min(lane, ntot - 1));
    for (int j0 = 0; j0 < nrows; j0 += 4) {
      float w[4], lse_out[4];
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        const int j = j0 + jj;
        const float ls = (lane < ntot && j < nrows)
                             ? __ldcg(slot_lse<kRec>(p, my_slot, src_row(lane, j)))
                             : -INFINITY;
        float mx = ls;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        const float mx_cur = (mx == -INFINITY) ? 0.f : mx;
        const float e = (lane < ntot) ? ex2(ls * kLog2e - mx_cur * kLog2e) : 0.f;
        float sum = e;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        lse_out[jj] = __logf(sum) + mx;
        const float inv = (sum == 0.f || sum != sum) ? 0.f : 1.f / sum;
        w[jj] = e * inv;
      }
      float4 acc[4];
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) acc[jj] = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int k = 0; k < ntot; ++k) {
        const int64_t sk = src_slot(k);
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          const float wk = __shfl_sync(0xffffffffu, w[jj], k);
          if (j0 + jj < nrows) {
            const float4 o =
                __ldcg(reinterpret_cast<const float4*>(slot_o<kRec>(p, sk, src_row(k, j0 + jj))) + lane);
            acc[jj].x += wk * o.x;
            acc[jj].y += wk * o.y;
            acc[jj].z += wk * o.z;
            acc[jj].w += wk * o.w;
          }
        }
      }
      __syncwarp();  // every lane's reads of these rows precede the writes
#pragma unroll
      for (int jj = 0; jj < 4; ++jj)
        if (j0 + jj < nrows) emit(j0 + jj, acc[jj], lse_out[jj]);
    }
    return;
  }
  // many sources: lane k owns sources k, k + 32, ...; still no load waits on
  // another's result within a phase.
  // Lane k owns sources k, k + 32, ...; every load of a phase is independent
  // of the others (an empty source has weight 0 and an all-zero partial, so
  // all sources are accumulated unconditionally).  Rows in chunks of 4 keep
  // the register footprint small.
  for (int j0 = 0; j0 < nrows; j0 += 4) {
    float w[4], lse_out[4];
    float mx_cur[4], inv[4];
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      const int j = j0 + jj;
      float mx = -INFINITY;
      if (j < nrows)
        for (int k = lane; k < ntot; k += 32)
          mx = fmaxf(mx, __ldcg(slot_lse<kRec>(p, src_slot(k), src_row(k, j))));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      mx_cur[jj] = (mx == -INFINITY) ? 0.f : mx;
      float sum = 0.f;
      if (j < nrows)
        for (int k = lane; k < ntot; k += 32)
          sum += ex2(__ldcg(slot_lse<kRec>(p, src_slot(k), src_row(k, j))) * kLog2e -
                     mx_cur[jj] * kLog2e);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      lse_out[jj] = __logf(sum) + mx;
      inv[jj] = (sum == 0.f || sum != sum) ? 0.f : 1.f / sum;
    }
    float4 acc[4];
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) acc[jj] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int k0 = 0; k0 < ntot; k0 += 32) {
      // weights of sources k0 .. k0 + 31, one per lane
      const int kl = k0 + lane;
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        const int j = j0 + jj;
        w[jj] = (kl < ntot && j < nrows)
                    ? ex2(__ldcg(slot_lse<kRec>(p, src_slot(kl), src_row(kl, j))) * kLog2e -
                          mx_cur[jj] * kLog2e) * inv[jj]
                    : 0.f;
      }
      const int kn = min(32, ntot - k0);
      for (int kk = 0; kk < kn; ++kk) {
        const int64_t sk = src_slot(k0 + kk);
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          const float wk = __shfl_sync(0xffffffffu, w[jj], kk);
          if (j0 + jj < nrows) {
            const float4 o = __ldcg(
                reinterpret_cast<const float4*>(slot_o<kRec>(p, sk, src_row(k0 + kk, j0 + jj))) + lane);
            acc[jj].x += wk * o.x;
            acc[jj].y += wk * o.y;
            acc[jj].z += wk * o.z;
            acc[jj].w += wk * o.w;
          }
        }
      }
    }
    __syncwarp();  // every lane's reads of these rows precede the writes
#pragma unroll
    for (int jj = 0; jj < 4; ++jj)
      if (j0 + jj < nrows) emit(j0 + jj, acc[jj], lse_out[jj]);
  }
}

template <int NT>
__host__ __device__ constexpr int decode_qslot_bytes() {
  return 8 * NT * kQRowBytes;
}

// Pages of one work unit.  An fp8 page-head is half the bytes of a 16-bit one
// and its per-page instruction stream (conversions, softmax, the MMA issue)
// sets the pace, so an fp8 unit is two consecutive pages of one (sequence, kv
// head): one stage holds both (8 KB, as a 16-bit page), one online-softmax
// update and one max/rescale cover 32 tokens, and the list, the stream-K cut
// and the split records count units.
template <bool kFP8>
__host__ __device__ constexpr int unit_pages() {
  return kFP8 ? 2 : 1;
}
// Stages per warp and their size.
template <bool kFP8, int kQNT>
__host__ __device__ constexpr int decode_stages() {
  return kFP8 ? kDecodeFp8Stages : kDecodeStages;
}
template <bool kFP8>
__host__ __device__ constexpr int decode_warps() {
  return kFP8 ? kDecodeFp8Warps : kDecodeWarps;
}
template <bool kFP8>
__host__ __device__ constexpr int decode_stage_bytes() {
  return kFP8 ? 4 * kBoxBytesF8 : kStageBytes;  // fp8: K page 0, K page 1, V page 0, V page 1
}

template <int kQNT, bool kFP8 = false>
__host__ __device__ constexpr int decode_smem_bytes_before_table() {
  // stages | per-warp query slots | mbarriers
  constexpr int D = decode_stages<kFP8, kQNT>();
  constexpr int W = decode_warps<kFP8>();
  return W * D * decode_stage_bytes<kFP8>() + W * D * decode_qslot_bytes<kQNT>() + W * D * 8;
}

// Own segment of sequence b (cascade modes): its split geometry in the list.
struct OwnSeg {
  int64_t slot0;  // slot of its first split
  int nsplit;
};
__device__ __forceinline__ OwnSeg own_segment(const Tables& tb, int b, int h, int Hkv) {
  const int P = seq_pages(tb.prefix, b);
  const int64_t seg0 = tb.pre_total + static_cast<int64_t>(tb.prefix[b]) * Hkv + static_cast<int64_t>(h) * P;
  const int64_t fw = warp_of(tb, seg0), lw = warp_of(tb, seg0 + P - 1);
  OwnSeg s;
  s.slot0 = fw + tb.pre_units + static_cast<int64_t>(b) * Hkv + h;
  s.nsplit = static_cast<int>(lw - fw + 1);
  return s;
}

// Slot holding the merged prefix result of member b of group g for kv head h,
// and the record row of its first query head.
__device__ __forceinline__ void prefix_result(const DecodeParams& p, const Tables& tb, int g, int b,
                                              int h, int Hkv, int64_t& slot, int& row0) {
  const int first = __ldg(p.cas_group_first + g);
  const int size = __ldg(p.cas_group_size + g);
  const int pages = __ldg(p.cas_group_pages + g);
  const int passes = (size + tb.mpp - 1) / tb.mpp;
  const int m = b - first;
  const int pass = m / tb.mpp;
  const int64_t seg0 = static_cast<int64_t>(tb.gph[g]) * Hkv + (static_cast<int64_t>(h) * passes + pass) * pages;
  const int64_t unit = static_cast<int64_t>(tb.gu[g]) * Hkv + static_cast<int64_t>(h) * passes + pass;
  slot = warp_of(tb, seg0) + unit;
  row0 = (m - pass * tb.mpp) * p.group;
}

// One warp streams page-heads [start, end) of one region of the list (plain
// list, cascade prefix region, or cascade own-segment region; indices are
// global list positions).  k0: ring uses so far by this warp.  Returns the ring
// uses after the range, or -1 after a wait timeout.
// Dim (within a 16-dim output tile) of accumulator row g (hi = 0) or g + 8
// (hi = 1): in order for 16-bit caches, (2g, 2g+1) for fp8 caches.
template <bool kFP8>
__device__ __forceinline__ int out_row(int g, int hi) {
  return kFP8 ? 2 * g + hi : g + 8 * hi;
}

// Fused head all-gather, segments one warp streams alone: the segment's
// output rows (o * inv rounded as the direct store rounds them) into every
// peer's slab.  For each 16-dim tile mi and half, the accumulators form an
// m8n8 b16 matrix with dims on rows and query heads on columns;
// movmatrix.trans hands lane (g, t) two dims of head g: 16-bit caches dims
// 16mi + 8 half + 2t, +1; fp8 caches (rows permuted, see out_row) dims
// 16mi + 4t, +2 and 16mi + 4t + 1, +3, interleaved into 4 consecutive dims.
// Each warp store then moves 16- (16-bit) or 32-byte (fp8) runs of 8 rows.
template <bool kBF16, bool kFP8, int NT>
__device__ __forceinline__ void push_rows_direct(const DecodeParams& p, const float (&o)[NT][8][4],
                                                 const float (&inv)[NT][2], int qrow, int h, int g,
                                                 int t, int lane) {
  if (qrow >= p.gather_tokens) {
    if (lane == 0) set_status(p.gather_status, PS_DEV_BAD_METADATA);
    return;
  }
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const bool ok = nt * 8 + g < p.group;  // this lane's head after the transpose
    const int64_t row = qrow * p.gather_row_st + static_cast<int64_t>(h * p.group + nt * 8 + g) * 256;
#pragma unroll
    for (int mi = 0; mi < 8; ++mi) {
      const uint32_t a = movmatrix_t(pack2<kBF16>(o[nt][mi][0] * inv[nt][0], o[nt][mi][1] * inv[nt][1]));
      const uint32_t b = movmatrix_t(pack2<kBF16>(o[nt][mi][2] * inv[nt][0], o[nt][mi][3] * inv[nt][1]));
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        char* dst = r < p.gather_world ? p.gather_rows[r] : nullptr;
        if (!ok || dst == nullptr) continue;
        if constexpr (kFP8) {
          *reinterpret_cast<uint2*>(dst + row + (16 * mi + 4 * t) * 2) =
              make_uint2(__byte_perm(a, b, 0x5410), __byte_perm(a, b, 0x7632));
        } else {
          *reinterpret_cast<uint32_t*>(dst + row + (16 * mi + 2 * t) * 2) = a;
          *reinterpret_cast<uint32_t*>(dst + row + (16 * mi + 8 + 2 * t) * 2) = b;
        }
      }
    }
  }
}

template <bool kBF16, int NT, int kRec, int kQNT, int kMode, bool kFP8 = false, bool kGather = false>
__device__ __forceinline__ int stream_range(const DecodeParams& p, const CUtensorMap* kmap,
                                            const CUtensorMap* vmap, const Tables& tb,
                                            int64_t start, int64_t end, int64_t gw,
                                            uint8_t* wsm, uint8_t* wq, uint64_t* wbar, int k0,
                                            int lane) {
  constexpr int D = decode_stages<kFP8, kQNT>();
  constexpr int SB = decode_stage_bytes<kFP8>();
  constexpr int kUP = unit_pages<kFP8>();        // pages per unit
  constexpr int kUnitTokens = kPageTokens * kUP;
  // MMA operand type: the model dtype, or f16 for an fp8 cache (e4m3 codes
  // convert to f16 exactly)
  constexpr bool kMathBF16 = kBF16 && !kFP8;
  const int Hkv = p.num_kv_heads;
  const int sub_per_block = p.block_size / kPageTokens;
  const int group = p.group;
  const int cnt = static_cast<int>(end - start);
  const int64_t base = (kMode == kCasSuffix) ? tb.pre_total : 0;
  // per-tensor cache scales (an fp8 cache's dequantization) fold into the
  // score scale (K) and the output normalisation (V)
  const float k_scale = p.k_scale ? __ldg(p.k_scale) : 1.f;
  const float v_scale = p.v_scale ? __ldg(p.v_scale) : 1.f;
  const float scale_log2 = p.scale_log2 * k_scale;

  if (k0 > 0) {
    // the ring and query slots were last read by this warp's generic-proxy
    // loads; order them before the async-proxy refills
    fence_proxy_async_smem();
    __syncwarp();
  }

  // ---- producer state: block-table entries cached 32 at a time --------------
  int bt_b = -1, bt_e0 = 0, bt_reg = 0;
  int pseg = 0;  // segments started on the producer side

  // Issue the TMA loads of page-head c into `stage` (warp-collective).
  // `seg_start`: c begins a segment for this warp -> also bring its query rows.
  // KV pages are read once: evict them from L2 first
  const uint64_t kv_policy = l2_policy_evict_first();
  auto issue = [&](int stage, const Cursor& c, bool seg_start) {
    const int pg = (c.p + c.off) * kUP;  // first page of the unit
    const int e = pg / sub_per_block;
    const int e_last = (pg + kUP - 1) / sub_per_block;
    if (c.b != bt_b || e < bt_e0 || e_last >= bt_e0 + 32) {
      bt_b = c.b;
      bt_e0 = e;
      const int idx = e + lane;
      bt_reg = idx < p.max_blocks_per_seq ? __ldg(p.block_table + c.b * p.bt_stride + idx) : 0;
    }
    int blk = __shfl_sync(0xffffffffu, bt_reg, e - bt_e0);
    int blk1 = 0;
    bool has1 = false;  // fp8: the unit's second page exists
    if constexpr (kFP8) {
      blk1 = __shfl_sync(0xffffffffu, bt_reg, e_last - bt_e0);
      has1 = true;
      if (c.p == c.P - 1) {  // only a sequence's last unit can hold one page
        const int L = max(__ldg(p.seq_lens + c.b), 0);
        const int npg = min((L + kPageTokens - 1) / kPageTokens, p.max_blocks_per_seq * sub_per_block);
        has1 = pg + 1 < npg;
      }
    }
    const int sub = pg - e * sub_per_block;
    uint8_t* dst = wsm + stage * SB;
    uint64_t* bar = wbar + stage;
    const int nrows = (kMode == kCasPrefix) ? c.ncols : group;
    const uint32_t qbytes = seg_start ? static_cast<uint32_t>(nrows) * (kHeadDim * 2) : 0u;
    if (lane == 0) {
      if (blk < 0 || blk >= p.num_blocks) {
        set_status(p.status, PS_DEV_BLOCK_OUT_OF_RANGE);
        blk = 0;
      }
      const int tok = sub * kPageTokens;
      if constexpr (kFP8) {
        // K page 0 | K page 1 | V page 0 | V page 1; a missing second page
        // leaves its boxes stale (every token of it is masked)
        mbar_arrive_expect_tx(bar, (has1 ? 4 : 2) * kBoxBytesF8 + qbytes);
        tma_load_4d_hint(dst, kmap, bar, 0, c.h, tok, blk, kv_policy);
        tma_load_4d_hint(dst + 2 * kBoxBytesF8, vmap, bar, 0, c.h, tok, blk, kv_policy);
        if (has1) {
          if (blk1 < 0 || blk1 >= p.num_blocks) {
            set_status(p.status, PS_DEV_BLOCK_OUT_OF_RANGE);
            blk1 = 0;
          }
          const int tok1 = (pg + 1 - e_last * sub_per_block) * kPageTokens;
          tma_load_4d_hint(dst + kBoxBytesF8, kmap, bar, 0, c.h, tok1, blk1, kv_policy);
          tma_load_4d_hint(dst + 3 * kBoxBytesF8, vmap, bar, 0, c.h, tok1, blk1, kv_policy);
        }
      } else {
        mbar_arrive_expect_tx(bar, SB + qbytes);
        tma_load_4d_hint(dst + 0 * kBoxBytes, kmap, bar, 0, c.h, tok, blk, kv_policy);
        tma_load_4d_hint(dst + 1 * kBoxBytes, kmap, bar, 64, c.h, tok, blk, kv_policy);
        tma_load_4d_hint(dst + 2 * kBoxBytes, vmap, bar, 0, c.h, tok, blk, kv_policy);
        tma_load_4d_hint(dst + 3 * kBoxBytes, vmap, bar, 64, c.h, tok, blk, kv_policy);
      }
    }
    if (seg_start) {
      __syncwarp();  // expect_tx is armed before the row copies complete_tx
      if (lane < nrows) {
        int seq = c.b, qh = c.h * group + lane;
        if constexpr (kMode == kCasPrefix) {
          // column lane -> (member, query head) of this pass
          const int mem = lane / group;
          seq = c.b + c.pass * tb.mpp + mem;
          qh = c.h * group + (lane - mem * group);
        }
        const int qrow = p.qsl ? __ldg(p.qsl + seq) : seq;
        const uint16_t* src = reinterpret_cast<const uint16_t*>(p.q) + qrow * p.q_st + qh * p.q_sh;
        bulk_load(wq + (pseg % D) * decode_qslot_bytes<kQNT>() + lane * kQRowBytes, src,
                  kHeadDim * 2, bar);
      }
      ++pseg;
    }
  };

  // pc always names the most recently issued page-head; cc the one consumed next.
  Cursor pc = cursor_at<kMode>(start - base, p, tb, Hkv);
  Cursor cc = pc;
  const int npre = min(cnt, D);
  for (int k = 0; k < npre; ++k) {
    if (k > 0) cursor_next<kMode>(pc, p, tb, Hkv);
    issue((k0 + k) % D, pc, k == 0 || pc.p == 0);
  }
  int issued = npre;

  const int g = lane >> 2;  // MMA row group
  const int t = lane & 3;   // MMA thread-in-group
  // per-lane ldmatrix row/chunk offsets
  const int k_mi = lane >> 3;
  const int k_row = (lane & 7) + ((k_mi & 1) << 3);
  const int k_chk = k_mi >> 1;
  const int v_row = (lane & 7) + ((k_mi >> 1) << 3);
  const int v_chk = k_mi & 1;

  uint32_t qf[NT][8][2];
  float o[NT][8][4];
  float m[NT][2], l[NT][2];
  int L = 0;
  int ncols = group;
  int cseg = 0;  // segments started on the consumer side
  // fused append: this lane's 16 bytes of the new key (lanes 0-15) or value
  // (lanes 16-31) row of the current segment's (sequence, kv head)
  const bool fused = (kMode != kCasPrefix) && p.new_key != nullptr;
  uint4 new_row = make_uint4(0u, 0u, 0u, 0u);
  int64_t new_slot = -1;

  for (int k = 0; k < cnt; ++k) {
    const int kr = k0 + k;
    const int stage = kr % D;
    const uint32_t phase = static_cast<uint32_t>((kr / D) & 1);
    uint8_t* st = wsm + stage * SB;
    if (!mbar_wait_bounded(wbar + stage, phase)) {
      if (lane == 0) set_status(p.status, PS_DEV_WAIT_TIMEOUT);
      // drain copies still in flight into this warp's ring, bounded
      for (int kk = k + 1; kk < issued; ++kk)
        if (!mbar_wait_bounded(wbar + (k0 + kk) % D, static_cast<uint32_t>(((k0 + kk) / D) & 1))) break;
      return -1;
    }

    // ---- segment start: query fragments from the slot, reset state ------------
    if (k == 0 || cc.p == 0) {
      if constexpr (kMode == kCasPrefix) {
        L = cc.P * kUnitTokens;  // shared pages are complete for every member
        ncols = cc.ncols;
      } else {
        L = __ldg(p.seq_lens + cc.b);
      }
      if (fused) {
        // fetch the new token's row now; it is written when the segment's last
        // page comes through this warp (the warp that owns that page)
        const int qrow = p.qsl ? __ldg(p.qsl + cc.b) : cc.b;
        new_slot = __ldg(p.slot_mapping + qrow);
        const int c = lane & 15;
        const uint16_t* src = lane < 16
            ? reinterpret_cast<const uint16_t*>(p.new_key) + qrow * p.nk_st + cc.h * p.nk_sh
            : reinterpret_cast<const uint16_t*>(p.new_value) + qrow * p.nv_st + cc.h * p.nv_sh;
        new_row = __ldg(reinterpret_cast<const uint4*>(src) + c);
      }
      const uint32_t qbase = smem_u32(wq + (cseg % D) * decode_qslot_bytes<kQNT>());
      ++cseg;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const bool ok = nt * 8 + g < ncols;
        if constexpr (kFP8) {
          // f16 B fragments with the reduction dims of each 16-dim step in
          // the order the fp8 K fragments arrive: k = 2t, 2t+1 -> dims 4t,
          // 4t+1 and k = 2t+8, 2t+9 -> dims 4t+2, 4t+3 (a permutation of the
          // dot product's terms, the same on both operands)
          const uint8_t* qrow = wq + (cseg - 1) % D * decode_qslot_bytes<kQNT>() + (nt * 8 + g) * kQRowBytes;
#pragma unroll
          for (int ks = 0; ks < 8; ++ks) {
            const uint2 w = *reinterpret_cast<const uint2*>(qrow + (16 * ks + 4 * t) * 2);
            const float2 lo = unpack2<kBF16>(w.x), hi = unpack2<kBF16>(w.y);
            qf[nt][ks][0] = ok ? pack2<false>(lo.x, lo.y) : 0u;
            qf[nt][ks][1] = ok ? pack2<false>(hi.x, hi.y) : 0u;
          }
        } else {
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            // matrices: heads nt*8..+7 x dims 32i + 8*(lane/8) .. +7
            const uint32_t addr = qbase + (nt * 8 + (lane & 7)) * kQRowBytes + (32 * i + 8 * k_mi) * 2;
            uint32_t r0, r1, r2, r3;
            ldsm_x4(addr, r0, r1, r2, r3);
            qf[nt][2 * i][0] = ok ? r0 : 0u;
            qf[nt][2 * i][1] = ok ? r1 : 0u;
            qf[nt][2 * i + 1][0] = ok ? r2 : 0u;
            qf[nt][2 * i + 1][1] = ok ? r3 : 0u;
          }
        }
#pragma unroll
        for (int mi = 0; mi < 8; ++mi)
#pragma unroll
          for (int c = 0; c < 4; ++c) o[nt][mi][c] = 0.f;
        m[nt][0] = m[nt][1] = -INFINITY;
        l[nt][0] = l[nt][1] = 0.f;
      }
    }

    const int valid = min(kUnitTokens, L - (cc.p + cc.off) * kUnitTokens);

    // ---- fused append: the sequence's last unit carries the new token -----
    if (fused && cc.p == cc.P - 1 && new_slot >= 0) {
      const int pos = L - 1;
      const int bidx = pos / p.block_size;
      const int64_t want = static_cast<int64_t>(__ldg(p.block_table + cc.b * p.bt_stride + bidx)) *
                               p.block_size + (pos - bidx * p.block_size);
      if (new_slot == want) {
        // write the row into this stage's copy of the page (K lanes 0-15, V 16-31)
        const int r = pos & (kPageTokens - 1);
        const int c = lane & 15;
        const int64_t blk = new_slot / p.block_size, off = new_slot - blk * p.block_size;
        if constexpr (kFP8) {
          // this lane's 8 elements (dims 8c..8c+7) as e4m3(x / scale), as
          // ps_kv_append_fp8 stores them, into page u of the unit
          const int u = (pos & (kUnitTokens - 1)) / kPageTokens;
          const uint2 q8 = quantize8_e4m3<kBF16>(new_row, lane < 16 ? k_scale : v_scale);
          *reinterpret_cast<uint2*>(st + (lane < 16 ? 0 : 2 * kBoxBytesF8) + u * kBoxBytesF8 + r * 128 +
                                    ((((c >> 1) ^ (r & 7)) << 4) | ((c & 1) << 3))) = q8;
          uint8_t* dst = reinterpret_cast<uint8_t*>(lane < 16 ? p.key_cache : p.value_cache) +
                         blk * p.c_sblock + off * p.c_sslot + cc.h * p.c_shead;
          reinterpret_cast<uint2*>(dst)[c] = q8;
        } else {
          const int part = (lane < 16 ? 0 : 2) + (c >> 3);  // K lo/hi, V lo/hi box
          *reinterpret_cast<uint4*>(st + part * kBoxBytes + r * 128 + (((c & 7) ^ (r & 7)) << 4)) = new_row;
          // and into the cache, as ps_kv_append would
          uint16_t* dst = reinterpret_cast<uint16_t*>(lane < 16 ? p.key_cache : p.value_cache) +
                          blk * p.c_sblock + off * p.c_sslot + cc.h * p.c_shead;
          reinterpret_cast<uint4*>(dst)[c] = new_row;
        }
      } else if (lane == 0) {
        set_status(p.status, PS_DEV_BAD_METADATA);
      }
      __syncwarp();
    }

    // ---- S^T = K Q^T (per page u of the unit) ----------------------------------
    float s[kUP][NT][4];
#pragma unroll
    for (int u = 0; u < kUP; ++u)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) s[u][nt][0] = s[u][nt][1] = s[u][nt][2] = s[u][nt][3] = 0.f;
    const uint32_t kbase = smem_u32(st);
    if constexpr (kFP8) {
      // one ldmatrix.x4 per two 16-dim steps: matrices (tokens 0-7 | 8-15) x
      // (chunk 2j | 2j+1); a lane receives 4 consecutive e4m3 dims 4t..4t+3
      // of token g (or g+8), converted to the f16 pairs (4t, 4t+1) and
      // (4t+2, 4t+3) that match the permuted query fragments
#pragma unroll
      for (int u = 0; u < kUP; ++u)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int chunk = 2 * j + k_chk;
          const uint32_t addr = kbase + u * kBoxBytesF8 + k_row * 128 + ((chunk ^ (k_row & 7)) << 4);
          uint32_t r0, r1, r2, r3;
          ldsm_x4(addr, r0, r1, r2, r3);
          uint32_t k0l, k0h, k1l, k1h, k2l, k2h, k3l, k3h;
          e4m3x4_to_f16x2x2(r0, k0l, k0h);
          e4m3x4_to_f16x2x2(r1, k1l, k1h);
          e4m3x4_to_f16x2x2(r2, k2l, k2h);
          e4m3x4_to_f16x2x2(r3, k3l, k3h);
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            mma_16816<false>(s[u][nt], k0l, k1l, k0h, k1h, qf[nt][2 * j][0], qf[nt][2 * j][1]);
            mma_16816<false>(s[u][nt], k2l, k3l, k2h, k3h, qf[nt][2 * j + 1][0], qf[nt][2 * j + 1][1]);
          }
        }
    } else {
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const int half = ks >> 2;
        const int chunk = ((ks & 3) << 1) + k_chk;
        const uint32_t addr = kbase + half * kBoxBytes + k_row * 128 + ((chunk ^ (k_row & 7)) << 4);
        uint32_t a0, a1, a2, a3;
        ldsm_x4(addr, a0, a1, a2, a3);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) mma_16816<kBF16>(s[0][nt], a0, a1, a2, a3, qf[nt][ks][0], qf[nt][ks][1]);
      }
    }

    // ---- online softmax (exp2 domain), one max/rescale per unit ---------------
    uint32_t pb[kUP][NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int u = 0; u < kUP; ++u) {
        const bool v0 = u * kPageTokens + g < valid, v1 = u * kPageTokens + g + 8 < valid;
        s[u][nt][0] = v0 ? s[u][nt][0] * scale_log2 : -INFINITY;
        s[u][nt][1] = v0 ? s[u][nt][1] * scale_log2 : -INFINITY;
        s[u][nt][2] = v1 ? s[u][nt][2] * scale_log2 : -INFINITY;
        s[u][nt][3] = v1 ? s[u][nt][3] * scale_log2 : -INFINITY;
      }
      float alpha[2];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        float mx = fmaxf(s[0][nt][j], s[0][nt][j + 2]);
#pragma unroll
        for (int u = 1; u < kUP; ++u) mx = fmaxf(mx, fmaxf(s[u][nt][j], s[u][nt][j + 2]));
        mx = warp_max_xor(mx, 0);
        const float mnew = fmaxf(m[nt][j], mx);
        alpha[j] = ex2(m[nt][j] - mnew);  // m = -inf -> 0
        m[nt][j] = mnew;
      }
#pragma unroll
      for (int u = 0; u < kUP; ++u) {
        const float p0 = ex2(s[u][nt][0] - m[nt][0]);
        const float p1 = ex2(s[u][nt][1] - m[nt][1]);
        const float p2 = ex2(s[u][nt][2] - m[nt][0]);
        const float p3 = ex2(s[u][nt][3] - m[nt][1]);
        if (u == 0) {
          l[nt][0] = l[nt][0] * alpha[0] + p0 + p2;
          l[nt][1] = l[nt][1] * alpha[1] + p1 + p3;
        } else {
          l[nt][0] += p0 + p2;
          l[nt][1] += p1 + p3;
        }
        pb[u][nt][0] = movmatrix_t(pack2<kMathBF16>(p0, p1));
        pb[u][nt][1] = movmatrix_t(pack2<kMathBF16>(p2, p3));
      }
      if (alpha[0] != 1.f || alpha[1] != 1.f) {
#pragma unroll
        for (int mi = 0; mi < 8; ++mi) {
          o[nt][mi][0] *= alpha[0];
          o[nt][mi][1] *= alpha[1];
          o[nt][mi][2] *= alpha[0];
          o[nt][mi][3] *= alpha[1];
        }
      }
    }

    // ---- O^T += V^T P^T ------------------------------------------------------
    const bool tail = valid < kUnitTokens;
    if constexpr (kFP8) {
      // ldmatrix.trans over byte pairs: a lane receives dims (2g, 2g+1) of
      // tokens (2t, 2t+1) [or 8+...]; one byte permute splits them into the
      // token pairs of dim 2g and of dim 2g+1, which become accumulator rows
      // g and g+8 (the output rows of each 16-dim tile are permuted; the
      // epilogue writes them back in order)
#pragma unroll
      for (int u = 0; u < kUP; ++u) {
        const uint32_t vbase = kbase + 2 * kBoxBytesF8 + u * kBoxBytesF8;
        const int vu = valid - u * kPageTokens;  // valid tokens of page u (may be <= 0)
        const bool z0 = 2 * t >= vu, z1 = 2 * t + 1 >= vu;
        const bool z2 = 2 * t + 8 >= vu, z3 = 2 * t + 9 >= vu;
        const uint32_t m01 = (z0 ? 0u : 0xffffu) | (z1 ? 0u : 0xffff0000u);
        const uint32_t m23 = (z2 ? 0u : 0xffffu) | (z3 ? 0u : 0xffff0000u);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int chunk = 2 * j + k_chk;
          const uint32_t addr = vbase + k_row * 128 + ((chunk ^ (k_row & 7)) << 4);
          uint32_t r0, r1, r2, r3;
          ldsm_x4_t(addr, r0, r1, r2, r3);
#pragma unroll
          for (int h2 = 0; h2 < 2; ++h2) {
            const uint32_t lo = __byte_perm(h2 ? r2 : r0, 0u, 0x3120);  // tokens 2t, 2t+1
            const uint32_t hi = __byte_perm(h2 ? r3 : r1, 0u, 0x3120);  // tokens 2t+8, 2t+9
            uint32_t a0, a1, a2, a3;
            e4m3x4_to_f16x2x2(lo, a0, a1);
            e4m3x4_to_f16x2x2(hi, a2, a3);
            if (tail) {  // stale rows past seq_len: P is 0 there, keep NaN codes out too
              a0 &= m01;
              a1 &= m01;
              a2 &= m23;
              a3 &= m23;
            }
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
              mma_16816<false>(o[nt][2 * j + h2], a0, a1, a2, a3, pb[u][nt][0], pb[u][nt][1]);
          }
        }
      }
    } else {
    const bool z0 = 2 * t >= valid, z1 = 2 * t + 1 >= valid;
    const bool z2 = 2 * t + 8 >= valid, z3 = 2 * t + 9 >= valid;
    const uint32_t vbase = kbase + 2 * kBoxBytes;
#pragma unroll
    for (int mi = 0; mi < 8; ++mi) {
      const int half = mi >> 2;
      const int chunk = ((mi & 3) << 1) + v_chk;
      const uint32_t addr = vbase + half * kBoxBytes + v_row * 128 + ((chunk ^ (v_row & 7)) << 4);
      uint32_t a0, a1, a2, a3;
      ldsm_x4_t(addr, a0, a1, a2, a3);
      if (tail) {  // stale rows past seq_len: P is 0 there, keep NaN garbage out too
        const uint32_t mlo0 = z0 ? 0u : 0xffffu, mhi0 = z1 ? 0u : 0xffff0000u;
        const uint32_t mlo1 = z2 ? 0u : 0xffffu, mhi1 = z3 ? 0u : 0xffff0000u;
        a0 &= (mlo0 | mhi0);
        a1 &= (mlo0 | mhi0);
        a2 &= (mlo1 | mhi1);
        a3 &= (mlo1 | mhi1);
      }
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) mma_16816<kBF16>(o[nt][mi], a0, a1, a2, a3, pb[0][nt][0], pb[0][nt][1]);
    }
    }
    __syncwarp();

    // ---- refill this stage with the page D ahead -------------------------------
    if (issued < cnt) {
      fence_proxy_async_smem();
      cursor_next<kMode>(pc, p, tb, Hkv);
      issue(stage, pc, pc.p == 0);
      ++issued;
    }

    // ---- segment end: finalize ------------------------------------------------
    const bool seg_end = (cc.p == cc.P - 1) || (k == cnt - 1);
    if (seg_end) {
      const int b = cc.b, h = cc.h;
      // list position of the segment's first page-head and its unit index
      int64_t seg0, unit;
      if constexpr (kMode == kCasPrefix) {
        seg0 = static_cast<int64_t>(tb.gph[cc.g]) * Hkv +
               (static_cast<int64_t>(h) * cc.passes + cc.pass) * cc.P;
        unit = static_cast<int64_t>(tb.gu[cc.g]) * Hkv + static_cast<int64_t>(h) * cc.passes + cc.pass;
      } else {
        seg0 = base + static_cast<int64_t>(tb.prefix[b]) * Hkv + static_cast<int64_t>(h) * cc.P;
        unit = tb.pre_units + static_cast<int64_t>(b) * Hkv + h;
      }
      // (plain list: every page-head costs 1, so the warp is position / quota)
      const int64_t first_w = kMode == kPlain ? seg0 / tb.Qc : warp_of(tb, seg0);
      const int64_t last_w = kMode == kPlain ? (seg0 + cc.P - 1) / tb.Qc : warp_of(tb, seg0 + cc.P - 1);
      const int nsplit = static_cast<int>(last_w - first_w + 1);
      // cascade: an own segment whose sequence has a group prefix always
      // writes a partial; the prefix arrives as one more split
      const bool member = (kMode == kCasSuffix) && cc.off > 0;
      float inv[NT][2], lse[NT][2];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const float lt = warp_sum_xor_4_8_16(l[nt][j]);
          const bool zero = (lt == 0.f) || (lt != lt);
          inv[nt][j] = zero ? 0.f : v_scale / lt;
          lse[nt][j] = zero ? -INFINITY : (m[nt][j] + __log2f(lt)) * 0.6931471805599453f;
        }
      if (kMode != kCasPrefix && nsplit == 1 && !member) {
        const int qrow = p.qsl ? __ldg(p.qsl + b) : b;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const int col = nt * 8 + 2 * t + j;
            if (col < group) {
              const int qh = h * group + col;
              const int64_t ob = qrow * p.o_st + qh * p.o_sh;
#pragma unroll
              for (int mi = 0; mi < 8; ++mi) {
                store_out2<kBF16>(p.out, ob + mi * 16 + out_row<kFP8>(g, 0), o[nt][mi][j] * inv[nt][j]);
                store_out2<kBF16>(p.out, ob + mi * 16 + out_row<kFP8>(g, 1), o[nt][mi][j + 2] * inv[nt][j]);
              }
              if (g == 0 && p.lse) p.lse[qh * p.lse_sh + qrow * p.lse_st] = lse[nt][j];
            }
          }
        if constexpr (kGather) push_rows_direct<kBF16, kFP8, NT>(p, o, inv, qrow, h, g, t, lane);
      } else {
        const int64_t slot = gw + unit;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const int col = nt * 8 + 2 * t + j;
            if (col < ncols) {  // the rows a combine reads: the segment's query columns
              float* po = slot_o<kRec>(p, slot, col);
#pragma unroll
              for (int mi = 0; mi < 8; ++mi) {
                po[mi * 16 + out_row<kFP8>(g, 0)] = o[nt][mi][j] * inv[nt][j];
                po[mi * 16 + out_row<kFP8>(g, 1)] = o[nt][mi][j + 2] * inv[nt][j];
              }
              if (g == 0) *slot_lse<kRec>(p, slot, col) = lse[nt][j];
            }
          }
        // release: the warp's partial is visible (gpu scope) before the count
        __syncwarp();
        if constexpr (kMode == kCasPrefix) {
          bool done = nsplit == 1;
          if (!done) {
            int last = 0;
            if (lane == 0) {
              const int old = atomic_add_release_gpu(p.pre_counters + unit, 1);
              last = (old == nsplit - 1);
              if (last) fence_acq_rel_gpu();
            }
            done = __shfl_sync(0xffffffffu, last, 0) != 0;
            __syncwarp();  // lane 0's acquire orders the whole warp's reads
            if (done) {
              // merge the prefix splits in place into the first split's record
              const int64_t s0 = first_w + unit;
              combine_rows<kBF16, kRec, true>(p, s0, nsplit, -1, 0, ncols, 0, 0, s0, lane);
              if (lane == 0) p.pre_counters[unit] = 0;
              __syncwarp();
            }
          }
          if (done) {
            // the prefix result is complete: count it into every member's
            // combine; the member whose count completes is merged here
            const int nmem = ncols / group;
            int lastm = 0;
            if (lane < nmem) {
              const int bm = b + cc.pass * tb.mpp + lane;
              const OwnSeg os = own_segment(tb, bm, h, Hkv);
              const int old = atomic_add_release_gpu(p.counters + bm * Hkv + h, 1);
              lastm = (old == os.nsplit);  // own splits + this prefix
              if (lastm) fence_acq_rel_gpu();
            }
            unsigned todo = __ballot_sync(0xffffffffu, lastm);
            __syncwarp();
            while (todo) {
              const int mm = __ffs(todo) - 1;
              todo &= todo - 1;
              const int bm = b + cc.pass * tb.mpp + mm;
              const OwnSeg os = own_segment(tb, bm, h, Hkv);
              combine_rows<kBF16, kRec, false>(p, os.slot0, os.nsplit, first_w + unit, mm * group,
                                               group, bm, h, 0, lane);
              if (lane == 0) p.counters[bm * Hkv + h] = 0;
            }
          }
        } else {
          const int total = nsplit + (member ? 1 : 0);
          int last = 0;
          if (lane == 0) {
            const int old = atomic_add_release_gpu(p.counters + b * Hkv + h, 1);
            last = (old == total - 1);
            if (last) fence_acq_rel_gpu();  // acquire the other splits' partials
          }
          last = __shfl_sync(0xffffffffu, last, 0);
          __syncwarp();  // lane 0's acquire orders the whole warp's reads
          if (last) {
            int64_t xslot = -1;
            int xrow0 = 0;
            if (member) prefix_result(p, tb, __ldg(p.cas_seq_group + b), b, h, Hkv, xslot, xrow0);
            combine_rows<kBF16, kRec, false>(p, first_w + unit, nsplit, xslot, xrow0, group, b, h, 0,
                                             lane);
            if (lane == 0) p.counters[b * Hkv + h] = 0;
          }
        }
      }
    }
    if (k + 1 < cnt) cursor_next<kMode>(cc, p, tb, Hkv);
  }
  return k0 + cnt;
}

// Exclusive scan over the block of one int per thread; *total gets the sum.
// s_warp: one int per warp of the block.  Contains __syncthreads.
__device__ __forceinline__ int block_exclusive_scan(int v, int* s_warp, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int u = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += u;
  }
  if (lane == 31) s_warp[warp] = incl;
  __syncthreads();
  int off = 0, tot = 0;
  const int nw = static_cast<int>(blockDim.x >> 5);
  for (int w = 0; w < nw; ++w) {
    const int x = s_warp[w];
    if (w < warp) off += x;
    tot += x;
  }
  __syncthreads();
  *total = tot;
  return off + incl - v;
}

__device__ __forceinline__ int own_pages_of(const DecodeParams& p, int b, int sub_per_block) {
  int qlen = 1;
  if (p.qsl) qlen = __ldg(p.qsl + b + 1) - __ldg(p.qsl + b);
  if (qlen != 1) return 0;
  const int L = __ldg(p.seq_lens + b);
  const int P = (max(L, 0) + kPageTokens - 1) / kPageTokens;
  return min(P, p.max_blocks_per_seq * sub_per_block);
}

// Fused head all-gather, after this CTA's streaming (the whole CTA).  Rows
// written: every CTA's peer stores precede its arrival (a system-scope fence
// per thread); the CTA that arrives last publishes "rows written" to every
// rank.  Each CTA then waits for every rank's flag and copies a share of the
// peers' rows from this rank's slab into gather_out; the last CTA to finish
// copying publishes "rows copied" and waits for every rank's, so that when
// the kernel completes no peer still needs the rows this rank will push in
// its next call.  All waits are bounded (status PS_DEV_WAIT_TIMEOUT).
__device__ __noinline__ void gather_tail(const DecodeParams& p) {
  char* own = p.gather_slab[p.gather_rank];
  const int32_t e = peer::call_epoch(own);
  __threadfence_system();
  if (peer::last_cta(own)) peer::signal(p.gather_slab, p.gather_world, p.gather_rank, 0, e);
  if (peer::wait_all(own, p.gather_world, 0, e, p.gather_status)) {
    const int hq = p.gather_hq_local;
    const int64_t row_vecs = static_cast<int64_t>(p.gather_world) * hq * 16;  // 16-byte vectors per token
    const int64_t peer_vecs = row_vecs - static_cast<int64_t>(hq) * 16;
    const int64_t nvec = static_cast<int64_t>(p.gather_tokens) * peer_vecs;
    const char* rows = own + kDecodeGatherRowsOffset;
    const int own_lo = p.gather_rank * hq;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < nvec;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
      const int64_t t = i / peer_vecs;
      const int rem = static_cast<int>(i - t * peer_vecs);
      const int c = rem & 15;
      const int hp = rem >> 4;
      const int hg = hp < own_lo ? hp : hp + hq;  // this rank's heads are already in gather_out
      const uint4 v = *reinterpret_cast<const uint4*>(rows + t * p.gather_row_st + hg * 256 + c * 16);
      *reinterpret_cast<uint4*>(p.gather_out + t * p.gather_o_st + hg * p.gather_o_sh + c * 16) = v;
    }
  }
  if (peer::last_cta(own, kDecodeGatherDone2Word)) {
    peer::signal(p.gather_slab, p.gather_world, p.gather_rank, 1, e);
    peer::wait_all(own, p.gather_world, 1, e, p.gather_status);
    peer::close_call(own, e);
  }
}

// kGather: the fused head all-gather is compiled in (plain decode only); the
// kernels without it carry none of its code
template <bool kBF16, int NT, bool kCascade, bool kFP8, bool kGather = false>
__global__ void __launch_bounds__(decode_warps<kFP8>() * 32, kDecodeCtasPerSm)
    paged_decode_kernel(const __grid_constant__ DecodeParams p,
                        const __grid_constant__ CUtensorMap kmap,
                        const __grid_constant__ CUtensorMap vmap) {
  constexpr int kQNT = kCascade ? kPrefixNT : NT;
  constexpr int D = decode_stages<kFP8, kQNT>();
  constexpr int SB = decode_stage_bytes<kFP8>();
  constexpr int kRec = kCascade ? 8 * kPrefixNT : 8 * NT;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte alignment for the 128B-swizzled TMA destinations.
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  constexpr int W = decode_warps<kFP8>();
  uint8_t* qslots = smem + W * D * SB;
  uint64_t* bars =
      reinterpret_cast<uint64_t*>(qslots + W * D * decode_qslot_bytes<kQNT>());
  int* prefix = reinterpret_cast<int*>(bars + W * D);
  __shared__ int s_warp_tot[W];

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int B = p.num_seqs;
  const int Hkv = p.num_kv_heads;
  const int sub_per_block = p.block_size / kPageTokens;

  if (tid == 0) {
    tma_prefetch_desc(&kmap);
    tma_prefetch_desc(&vmap);
  }
  if (lane == 0) {
    for (int s = 0; s < D; ++s) mbar_init(&bars[warp * D + s], 1);
    fence_mbar_init();
  }
  // Programmatic dependent launch: everything above overlaps the previous
  // kernel in the stream; global memory is read only after it completes.
  asm volatile("griddepcontrol.wait;" ::: "memory");

  Tables tb;
  tb.prefix = prefix;
  tb.soff = nullptr;
  tb.gph = nullptr;
  tb.gu = nullptr;
  tb.G = 0;
  tb.mpp = 1;
  tb.pre_total = 0;
  tb.pre_units = 0;
  tb.wp = 1;
  tb.wo = 1;
  tb.Qc = 1;

  // ---- prologue: units per sequence and their exclusive prefix sum ----------
  const int per = (B + blockDim.x - 1) / blockDim.x;
  const int b_lo = min(B, tid * per), b_hi = min(B, b_lo + per);
  int bad = 0;
  for (int b = b_lo; b < b_hi; ++b) {
    const int L = __ldg(p.seq_lens + b);
    int qlen = 1;
    if (p.qsl) qlen = __ldg(p.qsl + b + 1) - __ldg(p.qsl + b);
    if (qlen == 1) {
      if (L < 0) bad = 1;
      if ((max(L, 0) + kPageTokens - 1) / kPageTokens > p.max_blocks_per_seq * sub_per_block) bad = 1;
    } else if (qlen != 0) {
      bad = 1;  // multi-token queries belong to the prefill kernel
    }
  }

  int* soff = nullptr;
  int G = 0;
  if constexpr (kCascade) {
    // plan tables follow the sequence scan: soff[B], gph[Gmax+1], gu[Gmax+1]
    soff = prefix + B + 1;
    int* gph = soff + B;
    int* gu = gph + p.cas_max_groups + 1;
    G = min(max(__ldg(p.cas_num_groups), 0), p.cas_max_groups);
    tb.mpp = max(1, 16 / p.group);
    tb.wp = kCascadePrefixCost16;  // 16-column prefix pages cost more than own pages
    tb.wo = 16;
    // validate the plan; an invalid plan runs as a plain decode
    int bad_plan = tb.mpp < 2 && G > 0;
    for (int gi = tid; gi < G && !bad_plan; gi += blockDim.x) {
      const int f = __ldg(p.cas_group_first + gi), s = __ldg(p.cas_group_size + gi);
      const int pg = __ldg(p.cas_group_pages + gi);
      if (s < 2 || s > B || f < 0 || f > B - s || pg < 1 ||
          (gi > 0 && f < __ldg(p.cas_group_first + gi - 1) + __ldg(p.cas_group_size + gi - 1))) {
        bad_plan = 1;
        break;
      }
      for (int mm = 0; mm < s; ++mm) {
        const int b = f + mm;
        if (__ldg(p.cas_seq_group + b) != gi || own_pages_of(p, b, sub_per_block) - 1 < pg) {
          bad_plan = 1;
          break;
        }
      }
    }
    for (int b = b_lo; b < b_hi && !bad_plan; ++b) {
      const int gsb = __ldg(p.cas_seq_group + b);
      if (gsb >= G) bad_plan = 1;
      else if (gsb >= 0) {
        const int f = __ldg(p.cas_group_first + gsb);
        if (b < f || b >= f + __ldg(p.cas_group_size + gsb)) bad_plan = 1;
      }
    }
    if (__syncthreads_or(bad_plan)) {
      G = 0;
      bad = 1;
    }
    tb.soff = soff;
    tb.gph = gph;
    tb.gu = gu;
    tb.G = G;
    // group scans: pages * passes and passes
    const int gper = (G + blockDim.x - 1) / blockDim.x;
    const int g_lo = min(G, tid * gper), g_hi = min(G, g_lo + gper);
    int lph = 0, lu = 0;
    for (int gi = g_lo; gi < g_hi; ++gi) {
      const int passes = (__ldg(p.cas_group_size + gi) + tb.mpp - 1) / tb.mpp;
      lph += passes * __ldg(p.cas_group_pages + gi);
      lu += passes;
    }
    int tot_ph, tot_u;
    int run_ph = block_exclusive_scan(lph, s_warp_tot, &tot_ph);
    int run_u = block_exclusive_scan(lu, s_warp_tot, &tot_u);
    for (int gi = g_lo; gi < g_hi; ++gi) {
      gph[gi] = run_ph;
      gu[gi] = run_u;
      const int passes = (__ldg(p.cas_group_size + gi) + tb.mpp - 1) / tb.mpp;
      run_ph += passes * __ldg(p.cas_group_pages + gi);
      run_u += passes;
    }
    if (tid == 0) {
      gph[G] = tot_ph;
      gu[G] = tot_u;
    }
    tb.pre_total = static_cast<int64_t>(tot_ph) * Hkv;
    tb.pre_units = static_cast<int64_t>(tot_u) * Hkv;
  }

  // own units per sequence (after the group prefix in cascade mode)
  constexpr int kUP = unit_pages<kFP8>();
  int local = 0;
  for (int b = b_lo; b < b_hi; ++b) {
    int P = (own_pages_of(p, b, sub_per_block) + kUP - 1) / kUP;
    if constexpr (kCascade) {
      const int gsb = G > 0 ? __ldg(p.cas_seq_group + b) : -1;
      const int off = gsb >= 0 ? __ldg(p.cas_group_pages + gsb) : 0;
      soff[b] = off;
      P -= off;
    }
    local += P;
  }
  int total_own;
  int run = block_exclusive_scan(local, s_warp_tot, &total_own);
  for (int b = b_lo; b < b_hi; ++b) {
    prefix[b] = run;
    int P = (own_pages_of(p, b, sub_per_block) + kUP - 1) / kUP;
    if constexpr (kCascade) P -= soff[b];
    run += P;
  }
  if (tid == 0) prefix[B] = total_own;
  const int any_bad = __syncthreads_or(bad);
  if (tid == 0 && any_bad) set_status(p.status, PS_DEV_BAD_METADATA);

  const int64_t total = tb.pre_total + static_cast<int64_t>(total_own) * Hkv;
  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * W;
  const int64_t total_cost = list_cost(tb, total);
  tb.Qc = max(static_cast<int64_t>(max(tb.wp, tb.wo)),
              total_cost > 0 ? (total_cost + nwarps - 1) / nwarps : 1);

  // ---- empty sequences (q_len 1, seq_len 0): zero output, LSE -inf ----------
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + tid;
       i < static_cast<int64_t>(B) * p.num_q_heads; i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int b = static_cast<int>(i / p.num_q_heads);
    if (prefix[b + 1] != prefix[b]) continue;  // has pages: no global load needed
    const int qh = static_cast<int>(i - static_cast<int64_t>(b) * p.num_q_heads);
    int qlen = 1;
    if (p.qsl) qlen = __ldg(p.qsl + b + 1) - __ldg(p.qsl + b);
    if (qlen != 1) continue;
    const int qrow = p.qsl ? __ldg(p.qsl + b) : b;
    for (int d = 0; d < kHeadDim; ++d) store_out2<kBF16>(p.out, qrow * p.o_st + qh * p.o_sh + d, 0.f);
    if (p.lse) p.lse[qh * p.lse_sh + qrow * p.lse_st] = -INFINITY;
    if constexpr (kGather) {
      if (qrow < p.gather_tokens) {
        for (int r = 0; r < p.gather_world; ++r)
          if (p.gather_rows[r] != nullptr)
            for (int c = 0; c < 16; ++c)
              reinterpret_cast<uint4*>(p.gather_rows[r] + qrow * p.gather_row_st + qh * 256)[c] =
                  make_uint4(0u, 0u, 0u, 0u);
      } else {
        set_status(p.gather_status, PS_DEV_BAD_METADATA);
      }
    }
  }

  const int64_t gw = static_cast<int64_t>(blockIdx.x) * W + warp;
  const int64_t start = min(total, list_at_cost(tb, gw * tb.Qc));
  const int64_t end = min(total, list_at_cost(tb, (gw + 1) * tb.Qc));

  if (start < end) {
    uint8_t* wsm = smem + warp * D * SB;
    uint8_t* wq = qslots + warp * D * decode_qslot_bytes<kQNT>();
    uint64_t* wbar = bars + warp * D;

    if constexpr (kCascade) {
      int k = 0;
      if (start < tb.pre_total)
        k = stream_range<kBF16, kPrefixNT, kRec, kQNT, kCasPrefix>(
            p, &kmap, &vmap, tb, start, min(end, tb.pre_total), gw, wsm, wq, wbar, 0, lane);
      if (k >= 0 && end > tb.pre_total)
        stream_range<kBF16, NT, kRec, kQNT, kCasSuffix>(p, &kmap, &vmap, tb, max(start, tb.pre_total),
                                                        end, gw, wsm, wq, wbar, k, lane);
    } else {
      stream_range<kBF16, NT, kRec, kQNT, kPlain, kFP8, kGather>(p, &kmap, &vmap, tb, start, end, gw, wsm,
                                                                 wq, wbar, 0, lane);
    }
  }
  if constexpr (kGather) gather_tail(p);  // every warp of the CTA
}

template <bool kBF16, int NT, bool kCascade, bool kFP8 = false, bool kGather = false>
static int launch_t(const DecodeParams& p, const CUtensorMap& kmap, const CUtensorMap& vmap,
                    int sm_count, cudaStream_t stream) {
  constexpr int kQNT = kCascade ? kPrefixNT : NT;
  const int max_seqs = kCascade ? kCascadeMaxSeqs : kDecodeMaxSeqs;
  // sequence scan [B+1]; cascade adds soff[B] and two group scans [Gmax+1]
  auto table_ints = [](int B, int gmax) {
    return kCascade ? (2 * B + 1) + 2 * (gmax + 1) : B + 1;
  };
  const size_t smem = 1024 + decode_smem_bytes_before_table<kQNT, kFP8>() +
                      static_cast<size_t>(table_ints(p.num_seqs, p.cas_max_groups)) * 4;
  // the attribute is per function and per device
  static bool configured[64] = {false};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev >= 64) return static_cast<int>(cudaErrorInvalidDevice);
  if (!configured[dev]) {
    const cudaError_t e = cudaFuncSetAttribute(
        paged_decode_kernel<kBF16, NT, kCascade, kFP8, kGather>, cudaFuncAttributeMaxDynamicSharedMemorySize,
        static_cast<int>(1024 + decode_smem_bytes_before_table<kQNT, kFP8>() +
                         static_cast<size_t>(table_ints(max_seqs, max_seqs / 2)) * 4));
    if (e != cudaSuccess) return static_cast<int>(e);
    configured[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(sm_count * kDecodeCtasPerSm);
  cfg.blockDim = dim3(decode_warps<kFP8>() * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e =
      cudaLaunchKernelEx(&cfg, paged_decode_kernel<kBF16, NT, kCascade, kFP8, kGather>, p, kmap, vmap);
  return static_cast<int>(e != cudaSuccess ? e : cudaGetLastError());
}

}  // namespace ps

int64_t ps_decode_partial_slots(int num_seqs, int num_kv_heads, int sm_count, int cascade, int fp8) {
  // slot = global warp index + unit index; units: (sequence, kv head) and, in
  // cascade mode, at most one prefix segment per (sequence, kv head) more
  const int64_t units = static_cast<int64_t>(num_seqs) * num_kv_heads * (cascade ? 2 : 1);
  return static_cast<int64_t>(sm_count) * ps::kDecodeCtasPerSm *
             (fp8 ? ps::kDecodeFp8Warps : ps::kDecodeWarps) + units;
}

namespace ps {
// Plain decode (no cascade plan): cache dtype x I/O dtype x query-column tiles.
template <bool kGather>
static int launch_plain(const DecodeParams& p, const CUtensorMap& kmap, const CUtensorMap& vmap,
                        int dtype_bf16, int sm_count, cudaStream_t stream, int fp8_cache, int nt) {
  if (fp8_cache) {
    if (dtype_bf16)
      return nt == 1 ? launch_t<true, 1, false, true, kGather>(p, kmap, vmap, sm_count, stream)
                     : launch_t<true, 2, false, true, kGather>(p, kmap, vmap, sm_count, stream);
    return nt == 1 ? launch_t<false, 1, false, true, kGather>(p, kmap, vmap, sm_count, stream)
                   : launch_t<false, 2, false, true, kGather>(p, kmap, vmap, sm_count, stream);
  }
  if (dtype_bf16)
    return nt == 1 ? launch_t<true, 1, false, false, kGather>(p, kmap, vmap, sm_count, stream)
                   : launch_t<true, 2, false, false, kGather>(p, kmap, vmap, sm_count, stream);
  return nt == 1 ? launch_t<false, 1, false, false, kGather>(p, kmap, vmap, sm_count, stream)
                 : launch_t<false, 2, false, false, kGather>(p, kmap, vmap, sm_count, stream);
}
}  // namespace ps

int ps_launch_paged_decode(const ps::DecodeParams& p, const CUtensorMap& kmap,
                           const CUtensorMap& vmap, int dtype_bf16, int sm_count,
                           cudaStream_t stream, int fp8_cache) {
  const int nt = p.group <= 8 ? 1 : 2;
  if (p.cas_num_groups != nullptr && !fp8_cache && p.gather_world == 0) {
    // cascade: group <= 8 (checked by the caller)
    return dtype_bf16 ? ps::launch_t<true, 1, true>(p, kmap, vmap, sm_count, stream)
                      : ps::launch_t<false, 1, true>(p, kmap, vmap, sm_count, stream);
  }
  if (p.gather_world > 0)  // plain decode only (checked by the caller)
    return ps::launch_plain<true>(p, kmap, vmap, dtype_bf16, sm_count, stream, fp8_cache, nt);
  return ps::launch_plain<false>(p, kmap, vmap, dtype_bf16, sm_count, stream, fp8_cache, nt);
}
