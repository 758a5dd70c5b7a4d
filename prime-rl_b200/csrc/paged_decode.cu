// Paged split-KV decode attention for sm_100a, with the split combine fused.
//
// Semantics: vllm/vllm_flash_attn/cute/testing.py:326-455 (attention_ref: fp32
// softmax(q k^T * scale) v, GQA head groups, natural-log LSE) evaluated over the
// paged cache the way FA4 reads it (cute/paged_kv.py), with FA4's split-KV
// combine (cute/flash_fwd_combine.py:521-567 LSE merge, :633-640 weighted sum)
// and FA4's zero-sum guard (cute/softmax.py:147-158).
//
// Work decomposition ("stream-K" over page-heads):
//   A unit of work is one 16-token page of one KV head of one sequence.  The
//   page-heads of the batch are laid out in (sequence, kv head, page) order and
//   cut into equal contiguous ranges, one per warp of a persistent grid of one
//   CTA per SM.  A warp therefore streams an exactly equal share of the KV
//   bytes.  Where a warp's range crosses a (sequence, kv head) boundary it
//   finishes that segment as a split: it writes a normalised fp32 partial and
//   its LSE, bumps a per-(sequence, kv head) counter, and the warp that brings
//   the counter to the split count merges all partials (no waiting, so no
//   spin).  A segment that fits in one warp's range writes the output directly.
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
#include "ps_common.cuh"
#include "ps_launch.h"

namespace ps {

constexpr int kPageTokens = 16;
constexpr int kHeadDim = 128;
constexpr int kBoxBytes = kPageTokens * 64 * 2;  // 2 KB: 16 rows x 128 bytes
constexpr int kStageBytes = 4 * kBoxBytes;       // K lo, K hi, V lo, V hi
constexpr int kQRowBytes = kHeadDim * 2 + 16;    // padded query row (conflict-free ldmatrix)

// Split-slot record: kG output rows of 128 fp32, then kG fp32 LSEs.
template <int kG>
__device__ __forceinline__ float* slot_o(const DecodeParams& p, int64_t slot, int row) {
  return p.part + slot * (kG * (kHeadDim + 1)) + row * kHeadDim;
}
template <int kG>
__device__ __forceinline__ float* slot_lse(const DecodeParams& p, int64_t slot, int row) {
  return p.part + slot * (kG * (kHeadDim + 1)) + kG * kHeadDim + row;
}

struct Cursor {
  int b, h, p, P;  // sequence, kv head, page within sequence, pages of sequence
};

__device__ __forceinline__ int seq_pages(const int* prefix, int b) {
  return prefix[b + 1] - prefix[b];
}

// Advance to the next page-head in (sequence, kv head, page) order.
__device__ __forceinline__ void cursor_next(Cursor& c, const int* prefix, int num_kv_heads) {
  if (++c.p < c.P) return;
  c.p = 0;
  if (++c.h < num_kv_heads) return;
  c.h = 0;
  do {
    ++c.b;
    c.P = seq_pages(prefix, c.b);
  } while (c.P == 0);
}

// Locate page-head gi; requires gi < total.
__device__ __forceinline__ Cursor cursor_at(int64_t gi, const int* prefix, int num_seqs,
                                            int num_kv_heads) {
  int lo = 0, hi = num_seqs - 1;  // largest b with prefix[b]*Hkv <= gi
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (static_cast<int64_t>(prefix[mid]) * num_kv_heads <= gi)
      lo = mid;
    else
      hi = mid - 1;
  }
  Cursor c;
  c.b = lo;
  c.P = seq_pages(prefix, lo);
  const int64_t r = gi - static_cast<int64_t>(prefix[lo]) * num_kv_heads;
  c.h = static_cast<int>(r / c.P);
  c.p = static_cast<int>(r - static_cast<int64_t>(c.h) * c.P);
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

// Merge the n partials of segment (b, h) held in slots [slot0, slot0 + n).
// FA4 combine: lse_max over splits (0 if all -inf), scale_s =
// exp2((lse_s - lse_max_cur) * log2e), lse = log(sum) + lse_max, inv = 0 for a
// zero/NaN sum, O = sum_s scale_s * inv * O_s over splits with scale > 0.
template <bool kBF16, int NT>
__device__ __noinline__ void combine_segment(const DecodeParams& p, int b, int h, int64_t slot0,
                                             int n,
                                int lane) {
  constexpr int kG = 8 * NT;
  const int group = p.group;
  const int qrow = p.qsl ? __ldg(p.qsl + b) : b;
  const float kLog2e = 1.4426950408889634f;
  if (n <= 32) {
    // fast path: lane k owns split k; the loads of a phase are independent.
    // Heads in chunks of 4 keep the register footprint small.
    for (int j0 = 0; j0 < group; j0 += 4) {
      float w[4], lse_out[4];
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        const int j = j0 + jj;
        const float ls = (lane < n && j < group) ? __ldcg(slot_lse<kG>(p, slot0 + lane, j)) : -INFINITY;
        float mx = ls;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        const float mx_cur = (mx == -INFINITY) ? 0.f : mx;
        const float e = (lane < n) ? ex2(ls * kLog2e - mx_cur * kLog2e) : 0.f;
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
      // An empty split has weight 0 and an all-zero partial, so every split
      // can be accumulated unconditionally; the loads then do not wait for
      // the weights.
      for (int k = 0; k < n; ++k) {
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          const float wk = __shfl_sync(0xffffffffu, w[jj], k);
          if (j0 + jj < group) {
            const float4 o =
                __ldcg(reinterpret_cast<const float4*>(slot_o<kG>(p, slot0 + k, j0 + jj)) + lane);
            acc[jj].x += wk * o.x;
            acc[jj].y += wk * o.y;
            acc[jj].z += wk * o.z;
            acc[jj].w += wk * o.w;
          }
        }
      }
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        const int j = j0 + jj;
        if (j < group) {
          const int qh = h * group + j;
          const int64_t obase = qrow * p.o_st + qh * p.o_sh + lane * 4;
          uint2 packed;
          packed.x = pack2<kBF16>(acc[jj].x, acc[jj].y);
          packed.y = pack2<kBF16>(acc[jj].z, acc[jj].w);
          if constexpr (kBF16)
            *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(p.out) + obase) = packed;
          else
            *reinterpret_cast<uint2*>(reinterpret_cast<__half*>(p.out) + obase) = packed;
          if (lane == 0 && p.lse != nullptr) p.lse[qh * p.lse_sh + qrow * p.lse_st] = lse_out[jj];
        }
      }
    }
    return;
  }
  // general path: any number of splits
  for (int j = 0; j < group; ++j) {
    float mx = -INFINITY;
    for (int k = lane; k < n; k += 32) mx = fmaxf(mx, __ldcg(slot_lse<kG>(p, slot0 + k, j)));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const float mx_cur = (mx == -INFINITY) ? 0.f : mx;
    float sum = 0.f;
    for (int k = lane; k < n; k += 32)
      sum += ex2(__ldcg(slot_lse<kG>(p, slot0 + k, j)) * kLog2e - mx_cur * kLog2e);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    const float lse = __logf(sum) + mx;
    const float inv = (sum == 0.f || sum != sum) ? 0.f : 1.f / sum;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int k = 0; k < n; ++k) {
      const float w = ex2(__ldcg(slot_lse<kG>(p, slot0 + k, j)) * kLog2e - mx_cur * kLog2e) * inv;
      if (w > 0.f) {
        const float4 o = __ldcg(reinterpret_cast<const float4*>(slot_o<kG>(p, slot0 + k, j)) + lane);
        acc.x += w * o.x;
        acc.y += w * o.y;
        acc.z += w * o.z;
        acc.w += w * o.w;
      }
    }
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
  }
}

template <int NT>
__host__ __device__ constexpr int decode_qslot_bytes() {
  return 8 * NT * kQRowBytes;
}

template <int NT>
__host__ __device__ constexpr int decode_smem_bytes_before_table() {
  // stages | per-warp query slots | mbarriers
  return kDecodeWarps * kDecodeStages * kStageBytes +
         kDecodeWarps * kDecodeStages * decode_qslot_bytes<NT>() + kDecodeWarps * kDecodeStages * 8;
}

template <bool kBF16, int NT>
__global__ void __launch_bounds__(kDecodeWarps * 32, kDecodeCtasPerSm)
    paged_decode_kernel(const __grid_constant__ DecodeParams p,
                        const __grid_constant__ CUtensorMap kmap,
                        const __grid_constant__ CUtensorMap vmap) {
  constexpr int D = kDecodeStages;
  constexpr int kG = 8 * NT;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte alignment for the 128B-swizzled TMA destinations.
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* qslots = smem + kDecodeWarps * D * kStageBytes;
  uint64_t* bars =
      reinterpret_cast<uint64_t*>(qslots + kDecodeWarps * D * decode_qslot_bytes<NT>());
  int* prefix = reinterpret_cast<int*>(bars + kDecodeWarps * D);
  __shared__ int s_warp_tot[kDecodeWarps];

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

  // ---- prologue: pages per sequence and their exclusive prefix sum ----------
  const int per = (B + blockDim.x - 1) / blockDim.x;
  const int b_lo = min(B, tid * per), b_hi = min(B, b_lo + per);
  int local = 0;
  int bad = 0;
  for (int b = b_lo; b < b_hi; ++b) {
    int L = __ldg(p.seq_lens + b);
    int qlen = 1;
    if (p.qsl) qlen = __ldg(p.qsl + b + 1) - __ldg(p.qsl + b);
    int P = 0;
    if (qlen == 1) {
      if (L < 0) {
        L = 0;
        bad = 1;
      }
      P = (L + kPageTokens - 1) / kPageTokens;
      const int maxP = p.max_blocks_per_seq * sub_per_block;
      if (P > maxP) {
        P = maxP;
        bad = 1;
      }
    } else if (qlen != 0) {
      bad = 1;  // multi-token queries belong to the prefill kernel
    }
    local += P;
  }
  // block exclusive scan of `local`
  int incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) s_warp_tot[warp] = incl;
  const int any_bad = __syncthreads_or(bad);
  int warp_off = 0;
  for (int w = 0; w < warp; ++w) warp_off += s_warp_tot[w];
  int run = warp_off + incl - local;
  for (int b = b_lo; b < b_hi; ++b) {
    prefix[b] = run;
    const int L = __ldg(p.seq_lens + b);
    int qlen = 1;
    if (p.qsl) qlen = __ldg(p.qsl + b + 1) - __ldg(p.qsl + b);
    int P = 0;
    if (qlen == 1) {
      P = (max(L, 0) + kPageTokens - 1) / kPageTokens;
      P = min(P, p.max_blocks_per_seq * sub_per_block);
    }
    run += P;
  }
  if (tid == blockDim.x - 1) prefix[B] = warp_off + incl;  // last thread owns the tail
  __syncthreads();
  if (tid == 0 && any_bad) set_status(p.status, PS_DEV_BAD_METADATA);

  const int total_pages = prefix[B];
  const int64_t total = static_cast<int64_t>(total_pages) * Hkv;
  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * kDecodeWarps;
  const int64_t Q = total > 0 ? (total + nwarps - 1) / nwarps : 1;

  // ---- empty sequences (q_len 1, seq_len 0): zero output, LSE -inf ----------
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + tid;
       i < static_cast<int64_t>(B) * p.num_q_heads; i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int b = static_cast<int>(i / p.num_q_heads);
    const int qh = static_cast<int>(i - static_cast<int64_t>(b) * p.num_q_heads);
    int qlen = 1;
    if (p.qsl) qlen = __ldg(p.qsl + b + 1) - __ldg(p.qsl + b);
    if (qlen != 1 || prefix[b + 1] != prefix[b]) continue;
    const int qrow = p.qsl ? __ldg(p.qsl + b) : b;
    for (int d = 0; d < kHeadDim; ++d) store_out2<kBF16>(p.out, qrow * p.o_st + qh * p.o_sh + d, 0.f);
    if (p.lse) p.lse[qh * p.lse_sh + qrow * p.lse_st] = -INFINITY;
  }

  const int64_t gw = static_cast<int64_t>(blockIdx.x) * kDecodeWarps + warp;
  const int64_t start = gw * Q;
  const int64_t end = min(total, start + Q);
  if (start >= end) return;
  const int cnt = static_cast<int>(end - start);

  uint8_t* wsm = smem + warp * D * kStageBytes;
  uint8_t* wq = qslots + warp * D * decode_qslot_bytes<NT>();
  uint64_t* wbar = bars + warp * D;
  const int group = p.group;

  // ---- producer state: block-table entries cached 32 at a time --------------
  int bt_b = -1, bt_e0 = 0, bt_reg = 0;
  int pseg = 0;  // segments started on the producer side

  // Issue the TMA loads of page-head c into `stage` (warp-collective).
  // `seg_start`: c begins a segment for this warp -> also bring its query rows.
  auto issue = [&](int stage, const Cursor& c, bool seg_start) {
    const int e = c.p / sub_per_block;
    if (c.b != bt_b || e < bt_e0 || e >= bt_e0 + 32) {
      bt_b = c.b;
      bt_e0 = e;
      const int idx = e + lane;
      bt_reg = idx < p.max_blocks_per_seq ? __ldg(p.block_table + c.b * p.bt_stride + idx) : 0;
    }
    int blk = __shfl_sync(0xffffffffu, bt_reg, e - bt_e0);
    const int sub = c.p - e * sub_per_block;
    uint8_t* dst = wsm + stage * kStageBytes;
    uint64_t* bar = wbar + stage;
    const uint32_t qbytes = seg_start ? static_cast<uint32_t>(group) * (kHeadDim * 2) : 0u;
    if (lane == 0) {
      if (blk < 0 || blk >= p.num_blocks) {
        set_status(p.status, PS_DEV_BLOCK_OUT_OF_RANGE);
        blk = 0;
      }
      mbar_arrive_expect_tx(bar, kStageBytes + qbytes);
      const int tok = sub * kPageTokens;
      tma_load_4d(dst + 0 * kBoxBytes, &kmap, bar, 0, c.h, tok, blk);
      tma_load_4d(dst + 1 * kBoxBytes, &kmap, bar, 64, c.h, tok, blk);
      tma_load_4d(dst + 2 * kBoxBytes, &vmap, bar, 0, c.h, tok, blk);
      tma_load_4d(dst + 3 * kBoxBytes, &vmap, bar, 64, c.h, tok, blk);
    }
    if (seg_start) {
      __syncwarp();  // expect_tx is armed before the row copies complete_tx
      if (lane < group) {
        const int qrow = p.qsl ? __ldg(p.qsl + c.b) : c.b;
        const uint16_t* src = reinterpret_cast<const uint16_t*>(p.q) + qrow * p.q_st +
                              (c.h * group + lane) * p.q_sh;
        bulk_load(wq + (pseg % D) * decode_qslot_bytes<NT>() + lane * kQRowBytes, src,
                  kHeadDim * 2, bar);
      }
      ++pseg;
    }
  };

  const int* cprefix = prefix;
  // pc always names the most recently issued page-head; cc the one consumed next.
  Cursor pc = cursor_at(start, cprefix, B, Hkv);
  Cursor cc = pc;
  const int npre = min(cnt, D);
  for (int k = 0; k < npre; ++k) {
    if (k > 0) cursor_next(pc, cprefix, Hkv);
    issue(k, pc, k == 0 || pc.p == 0);
  }
  int issued = npre;

  const int g = lane >> 2;  // MMA row group
  const int t = lane & 3;   // MMA thread-in-group
  // per-lane ldmatrix row/chunk offsets (see header comment)
  const int k_mi = lane >> 3;
  const int k_row = (lane & 7) + ((k_mi & 1) << 3);
  const int k_chk = k_mi >> 1;
  const int v_row = (lane & 7) + ((k_mi >> 1) << 3);
  const int v_chk = k_mi & 1;

  uint32_t qf[NT][8][2];
  float o[NT][8][4];
  float m[NT][2], l[NT][2];
  int L = 0;
  int cseg = 0;  // segments started on the consumer side
  // fused append: this lane's 16 bytes of the new key (lanes 0-15) or value
  // (lanes 16-31) row of the current segment's (sequence, kv head)
  const bool fused = p.new_key != nullptr;
  uint4 new_row = make_uint4(0u, 0u, 0u, 0u);
  int64_t new_slot = -1;

  for (int k = 0; k < cnt; ++k) {
    const int stage = k % D;
    const uint32_t phase = static_cast<uint32_t>((k / D) & 1);
    uint8_t* st = wsm + stage * kStageBytes;
    if (!mbar_wait_bounded(wbar + stage, phase)) {
      if (lane == 0) set_status(p.status, PS_DEV_WAIT_TIMEOUT);
      // drain copies still in flight into this warp's ring, bounded
      for (int kk = k + 1; kk < issued; ++kk)
        if (!mbar_wait_bounded(wbar + kk % D, static_cast<uint32_t>((kk / D) & 1))) break;
      return;
    }

    // ---- segment start: query fragments from the slot, reset state ------------
    if (k == 0 || cc.p == 0) {
      L = __ldg(p.seq_lens + cc.b);
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
      const uint32_t qbase = smem_u32(wq + (cseg % D) * decode_qslot_bytes<NT>());
      ++cseg;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const bool ok = nt * 8 + g < group;
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
#pragma unroll
        for (int mi = 0; mi < 8; ++mi)
#pragma unroll
          for (int c = 0; c < 4; ++c) o[nt][mi][c] = 0.f;
        m[nt][0] = m[nt][1] = -INFINITY;
        l[nt][0] = l[nt][1] = 0.f;
      }
    }

    const int valid = min(kPageTokens, L - cc.p * kPageTokens);

    // ---- fused append: the sequence's last page carries the new token -----
    if (fused && cc.p == cc.P - 1 && new_slot >= 0) {
      const int pos = L - 1;
      const int bidx = pos / p.block_size;
      const int64_t want = static_cast<int64_t>(__ldg(p.block_table + cc.b * p.bt_stride + bidx)) *
                               p.block_size + (pos - bidx * p.block_size);
      if (new_slot == want) {
        // write the row into this stage's copy of the page (K lanes 0-15, V 16-31)
        const int r = pos & (kPageTokens - 1);
        const int c = lane & 15;
        const int part = (lane < 16 ? 0 : 2) + (c >> 3);  // K lo/hi, V lo/hi box
        *reinterpret_cast<uint4*>(st + part * kBoxBytes + r * 128 + (((c & 7) ^ (r & 7)) << 4)) = new_row;
        // and into the cache, as ps_kv_append would
        const int64_t blk = new_slot / p.block_size, off = new_slot - blk * p.block_size;
        uint16_t* dst = reinterpret_cast<uint16_t*>(lane < 16 ? p.key_cache : p.value_cache) +
                        blk * p.c_sblock + off * p.c_sslot + cc.h * p.c_shead;
        reinterpret_cast<uint4*>(dst)[c] = new_row;
      } else if (lane == 0) {
        set_status(p.status, PS_DEV_BAD_METADATA);
      }
      __syncwarp();
    }

    // ---- S^T = K Q^T -----------------------------------------------------------
    float s[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
    const uint32_t kbase = smem_u32(st);
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      const int half = ks >> 2;
      const int chunk = ((ks & 3) << 1) + k_chk;
      const uint32_t addr = kbase + half * kBoxBytes + k_row * 128 + ((chunk ^ (k_row & 7)) << 4);
      uint32_t a0, a1, a2, a3;
      ldsm_x4(addr, a0, a1, a2, a3);
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) mma_16816<kBF16>(s[nt], a0, a1, a2, a3, qf[nt][ks][0], qf[nt][ks][1]);
    }

    // ---- online softmax (exp2 domain) ----------------------------------------
    const bool v0 = g < valid, v1 = (g + 8) < valid;
    uint32_t pb[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      s[nt][0] = v0 ? s[nt][0] * p.scale_log2 : -INFINITY;
      s[nt][1] = v0 ? s[nt][1] * p.scale_log2 : -INFINITY;
      s[nt][2] = v1 ? s[nt][2] * p.scale_log2 : -INFINITY;
      s[nt][3] = v1 ? s[nt][3] * p.scale_log2 : -INFINITY;
      float alpha[2];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        float mx = fmaxf(s[nt][j], s[nt][j + 2]);
        mx = warp_max_xor(mx, 0);
        const float mnew = fmaxf(m[nt][j], mx);
        alpha[j] = ex2(m[nt][j] - mnew);  // m = -inf -> 0
        m[nt][j] = mnew;
      }
      const float p0 = ex2(s[nt][0] - m[nt][0]);
      const float p1 = ex2(s[nt][1] - m[nt][1]);
      const float p2 = ex2(s[nt][2] - m[nt][0]);
      const float p3 = ex2(s[nt][3] - m[nt][1]);
      l[nt][0] = l[nt][0] * alpha[0] + p0 + p2;
      l[nt][1] = l[nt][1] * alpha[1] + p1 + p3;
      if (alpha[0] != 1.f || alpha[1] != 1.f) {
#pragma unroll
        for (int mi = 0; mi < 8; ++mi) {
          o[nt][mi][0] *= alpha[0];
          o[nt][mi][1] *= alpha[1];
          o[nt][mi][2] *= alpha[0];
          o[nt][mi][3] *= alpha[1];
        }
      }
      pb[nt][0] = movmatrix_t(pack2<kBF16>(p0, p1));
      pb[nt][1] = movmatrix_t(pack2<kBF16>(p2, p3));
    }

    // ---- O^T += V^T P^T ------------------------------------------------------
    const uint32_t vbase = kbase + 2 * kBoxBytes;
    const bool tail = valid < kPageTokens;
    const bool z0 = 2 * t >= valid, z1 = 2 * t + 1 >= valid;
    const bool z2 = 2 * t + 8 >= valid, z3 = 2 * t + 9 >= valid;
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
      for (int nt = 0; nt < NT; ++nt) mma_16816<kBF16>(o[nt][mi], a0, a1, a2, a3, pb[nt][0], pb[nt][1]);
    }
    __syncwarp();

    // ---- refill this stage with the page D ahead -------------------------------
    if (issued < cnt) {
      fence_proxy_async_smem();
      cursor_next(pc, cprefix, Hkv);
      issue(stage, pc, pc.p == 0);
      ++issued;
    }

    // ---- segment end: finalize ------------------------------------------------
    const bool seg_end = (cc.p == cc.P - 1) || (k == cnt - 1);
    if (seg_end) {
      const int b = cc.b, h = cc.h;
      const int64_t seg0 = (static_cast<int64_t>(cprefix[b]) * Hkv + static_cast<int64_t>(h) * cc.P);
      const int64_t first_w = seg0 / Q;
      const int64_t last_w = (seg0 + cc.P - 1) / Q;
      const int nsplit = static_cast<int>(last_w - first_w + 1);
      const int qrow = p.qsl ? __ldg(p.qsl + b) : b;
      float inv[NT][2], lse[NT][2];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const float lt = warp_sum_xor_4_8_16(l[nt][j]);
          const bool zero = (lt == 0.f) || (lt != lt);
          inv[nt][j] = zero ? 0.f : 1.f / lt;
          lse[nt][j] = zero ? -INFINITY : (m[nt][j] + __log2f(lt)) * 0.6931471805599453f;
        }
      if (nsplit == 1) {
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
                store_out2<kBF16>(p.out, ob + mi * 16 + g, o[nt][mi][j] * inv[nt][j]);
                store_out2<kBF16>(p.out, ob + mi * 16 + g + 8, o[nt][mi][j + 2] * inv[nt][j]);
              }
              if (g == 0 && p.lse) p.lse[qh * p.lse_sh + qrow * p.lse_st] = lse[nt][j];
            }
          }
      } else {
        const int64_t slot = gw + static_cast<int64_t>(b) * Hkv + h;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const int col = nt * 8 + 2 * t + j;
            float* po = slot_o<kG>(p, slot, col);
#pragma unroll
            for (int mi = 0; mi < 8; ++mi) {
              po[mi * 16 + g] = o[nt][mi][j] * inv[nt][j];
              po[mi * 16 + g + 8] = o[nt][mi][j + 2] * inv[nt][j];
            }
            if (g == 0) *slot_lse<kG>(p, slot, col) = lse[nt][j];
          }
        // release: the warp's partial is visible (gpu scope) before the count
        __syncwarp();
        int last = 0;
        if (lane == 0) {
          const int old = atomic_add_release_gpu(p.counters + b * Hkv + h, 1);
          last = (old == nsplit - 1);
          if (last) fence_acq_rel_gpu();  // acquire the other splits' partials
        }
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last) {
          combine_segment<kBF16, NT>(p, b, h, first_w + static_cast<int64_t>(b) * Hkv + h, nsplit, lane);
          if (lane == 0) p.counters[b * Hkv + h] = 0;
        }
      }
    }
    if (k + 1 < cnt) cursor_next(cc, cprefix, Hkv);
  }
}

template <bool kBF16, int NT>
static int launch_t(const DecodeParams& p, const CUtensorMap& kmap, const CUtensorMap& vmap,
                    int sm_count, cudaStream_t stream) {
  const size_t smem = 1024 + decode_smem_bytes_before_table<NT>() + static_cast<size_t>(p.num_seqs + 1) * 4;
  // the attribute is per function and per device
  static bool configured[64] = {false};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev >= 64) return static_cast<int>(cudaErrorInvalidDevice);
  if (!configured[dev]) {
    const cudaError_t e = cudaFuncSetAttribute(
        paged_decode_kernel<kBF16, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
        static_cast<int>(1024 + decode_smem_bytes_before_table<NT>() + (kDecodeMaxSeqs + 1) * 4));
    if (e != cudaSuccess) return static_cast<int>(e);
    configured[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(sm_count * kDecodeCtasPerSm);
  cfg.blockDim = dim3(kDecodeWarps * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, paged_decode_kernel<kBF16, NT>, p, kmap, vmap);
  return static_cast<int>(e != cudaSuccess ? e : cudaGetLastError());
}

}  // namespace ps

int64_t ps_decode_partial_slots(int num_seqs, int num_kv_heads, int sm_count) {
  // slot = global warp index + (sequence * kv heads + kv head)
  return static_cast<int64_t>(sm_count) * ps::kDecodeCtasPerSm * ps::kDecodeWarps +
         static_cast<int64_t>(num_seqs) * num_kv_heads;
}

int ps_launch_paged_decode(const ps::DecodeParams& p, const CUtensorMap& kmap,
                           const CUtensorMap& vmap, int dtype_bf16, int sm_count,
                           cudaStream_t stream) {
  const int nt = p.group <= 8 ? 1 : 2;
  if (dtype_bf16) {
    return nt == 1 ? ps::launch_t<true, 1>(p, kmap, vmap, sm_count, stream)
                   : ps::launch_t<true, 2>(p, kmap, vmap, sm_count, stream);
  }
  return nt == 1 ? ps::launch_t<false, 1>(p, kmap, vmap, sm_count, stream)
                 : ps::launch_t<false, 2>(p, kmap, vmap, sm_count, stream);
}
