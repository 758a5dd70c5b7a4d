// Chunked-prefill paged attention on the sm_100a tensor cores (tcgen05 + TMEM).
//
// Semantics: vllm/vllm_flash_attn/cute/testing.py:326-455 (attention_ref) with
// causal=True, bottom-right aligned: in a sequence of seq_len L with q_len new
// query rows, query row i sees keys j <= L - q_len + i (construct_local_mask,
// testing.py:278-279).  Output bf16/fp16, natural-log LSE as FA4's
// softmax.finalize (cute/softmax.py:147-158).
//
// Tiling.  An M tile is 128 rows of (token, q head) pairs of ONE kv head: the
// GQA group is packed along M (row = token * group + head_in_group), so a KV
// tile loaded once serves every q head that reads it.  A CTA works on a PAIR of
// consecutive M tiles (A, B) of the same (sequence, kv head), so every KV tile
// it loads feeds two 128x128 products.  A KV tile is 128 keys = 8 pages of 16
// tokens gathered through the block table, one TMA box per page and 64-dim
// half, 128-byte swizzled (the canonical K-major SW128 layout for K; for V the
// same bytes are the MN-major SW128 layout of the PV B operand).
//
// Warp roles (384 threads, one persistent CTA per SM):
//   warp 0       TMA producer: Q tiles A and B, K/V tiles
//   warp 1       TMEM owner; lane 0 issues tcgen05.mma (M128 N128 K16) in the
//                order S_A(j) S_B(j) PV_A(j) S_A(j+1) PV_B(j) S_B(j+1) ...,
//                so each softmax group has two MMAs of the other tile to hide in
//   warps 2-3    idle (keep the softmax groups warpgroup-aligned)
//   warps 4-7    softmax + epilogue of tile A, warps 8-11 of tile B: one
//                thread per TMEM lane (= M row); S is read twice from TMEM
//                (row max, then exp2 + bf16 pack chunk by chunk) and P is
//                written over the S columns already read, as the A operand of
//                the PV product.  Online softmax in the exp2 domain with lazy
//                rescaling (the running max moves only when a tile's max
//                exceeds it by more than 2^8; O in TMEM is rescaled then).
// TMEM: S_A [0,128) S_B [128,256) O_A [256,384) O_B [384,512).
//
// Every mbarrier wait is bounded (~1 s); on timeout the kernel records
// PS_DEV_WAIT_TIMEOUT, raises a CTA-wide abort flag that ends every role's
// loop, and still frees its TMEM.
#include <climits>

#include "ps_common.cuh"
#include "ps_launch.h"
#include "tcgen05.cuh"

namespace ps {

constexpr int kKeys = 128;                    // keys per KV tile
constexpr int kRegionBytes = 128 * 128;       // [128 rows][64 x 16-bit], 128B swizzled
constexpr int kTileBytes = 2 * kRegionBytes;  // both 64-dim halves
constexpr int kKvStages = 2;
constexpr int kThreads = 384;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

// Of every 8 exponentials in a softmax row, this many are evaluated on the FMA
// pipe (exp2_fma) instead of the MUFU unit (16 results per clock per SM),
// which sets the length of a softmax step when both warpgroups exponentiate
// the same tile.  The macro exists for sweeps.
#ifndef PS_PREFILL_EMU_PER8
#define PS_PREFILL_EMU_PER8 1
#endif

// 2^x on the FMA/ALU pipes: 2^x = 2^n * 2^f with n = round(x) and
// f = x - n in [-0.5, 0.5]; 2^f by a cubic fitted for minimum relative error
// on that interval (Lawson-weighted least squares; max relative error 7.5e-5,
// far below the 2^-9 rounding of the bf16 P it feeds).  n is read from the
// mantissa of x + 1.5*2^23 and added to the exponent field.  x < -126
// (including -inf) returns 0, as ex2 of a masked score must.
__device__ __forceinline__ float exp2_fma(float x) {
  const float xc = fmaxf(x, -127.f);
  const float t = xc + 12582912.f;
  const float f = xc - (t - 12582912.f);
  const float p = fmaf(fmaf(fmaf(0.05517132f, f, 0.24261054f), f, 0.69326097f), f, 0.99992812f);
  const int n = __float_as_int(t) - 0x4B400000;
  const float r = __int_as_float(__float_as_int(p) + (n << 23));
  return x < -126.f ? 0.f : r;
}

// Packed fp32 pairs (sm_100 f32x2 instructions): one instruction updates two
// softmax elements.  Results equal two scalar fmaf / additions.
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
// Three-input maximum (sm_100); like fmaxf, a NaN input is ignored.
__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

struct PrefillSmem {
  // all tiles 1024-byte aligned (offsets from the aligned base)
  static constexpr int q_off = 0;  // Q_A then Q_B
  static constexpr int k_off = q_off + 2 * kTileBytes;
  static constexpr int v_off = k_off + kKvStages * kTileBytes;
  static constexpr int bar_off = v_off + kKvStages * kTileBytes;
  static constexpr int n_bars = 4 /*unit_full, unit_empty*/ + 2 /*q*/ + 4 * kKvStages /*kfull vfull kempty vempty*/ +
                                2 /*s_full*/ + 2 /*p_full*/ + 2 /*pv_done*/ + 2 /*mx_full*/ + 1 /*ep_full*/;
  static constexpr int misc_off = bar_off + n_bars * 8;  // tmem base, abort flag, next units[2]
  // row maxima and sums of the two halves of every row: [tile][half][row] fp32
  static constexpr int xchg_off = misc_off + 16;
  static constexpr int table_off = xchg_off + 2 * (2 * 2 * 128 * 4);
  static constexpr int bytes_before_table = table_off;
};

struct PBars {
  uint64_t* q_full;
  uint64_t* q_empty;
  uint64_t* kfull;    // [kKvStages]
  uint64_t* vfull;    // [kKvStages]
  uint64_t* kempty;   // [kKvStages]: both S products of the stage's K tile completed
  uint64_t* vempty;   // [kKvStages]: both PV products of the stage's V tile completed
  uint64_t* s_full;   // [2]: tile A, tile B
  uint64_t* p_full;   // [2]
  uint64_t* pv_done;  // [2]
  uint64_t* unit_full;   // [2]: a claimed unit id is in s_unit[k]
  uint64_t* unit_empty;  // [2]: every consumer has read s_unit[k]
  uint64_t* mx_full;     // [2]: both halves' row maxima of tile A / B are in s_mx
  uint64_t* ep_full;     // both halves' row sums of the unit are in s_l
};

// Consumers of the MMA warp (one thread) and the 8 softmax warps release a
// published unit id.
constexpr int kUnitConsumers = 1 + 8;

struct UnitInfo {
  int b, h;         // sequence, kv head
  int t0;           // first token (within the q chunk) of tile A; tile B starts at t0 + tpt
  int qlen, qrow0;  // query rows of the sequence, first global q row
  int ctx;          // L - q_len
  int kv_end;       // keys [0, kv_end) are visible to some row of the pair
  int ntiles;
};

// Units are (sequence, M-tile pair, kv head); within a sequence the pairs are
// enumerated from the last (longest causal range) to the first.
__device__ __forceinline__ UnitInfo unit_info(const PrefillParams& p, const int* prefix, int u) {
  UnitInfo ui;
  const int pu = u / p.num_kv_heads;
  ui.h = u - pu * p.num_kv_heads;
  int lo = 0, hi = p.num_seqs - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (prefix[mid] <= pu) lo = mid; else hi = mid - 1;
  }
  ui.b = lo;
  const int npairs = prefix[lo + 1] - prefix[lo];
  const int mp = npairs - 1 - (pu - prefix[lo]);
  ui.qrow0 = __ldg(p.qsl + lo);
  ui.qlen = __ldg(p.qsl + lo + 1) - ui.qrow0;
  const int L = __ldg(p.seq_lens + lo);
  ui.ctx = L - ui.qlen;
  ui.t0 = mp * 2 * p.tokens_per_tile;
  const int t1 = min(ui.qlen, ui.t0 + 2 * p.tokens_per_tile);
  ui.kv_end = ui.ctx + t1;
  ui.ntiles = (ui.kv_end + kKeys - 1) / kKeys;
  return ui;
}

// bounded wait that also observes the CTA abort flag; returns false to abort
__device__ __forceinline__ bool pwait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                      int32_t* status) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (clock64() - t0 > kWaitLimitCycles) {
      *abort_flag = 1;
      set_status(status, PS_DEV_WAIT_TIMEOUT);
      return false;
    }
  }
}

__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cta.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tmem_st_x16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

// Unit scheduling.  Static: CTA c takes units c, c + grid, ...  Dynamic
// (p.sched): CTA c starts with unit c; when its TMA warp has issued every
// load of its uit-th unit it claims the next id (grid + an atomic counter)
// and publishes it in s_unit[(uit + 1) & 1] (use m = uit >> 1 of that slot);
// the MMA thread and the softmax warps read it there.  Ids are claimed in unit
// order (longest pair of each sequence first), so the CTAs that finish early
// take the remaining units.
__device__ __forceinline__ int claim_and_publish(const PrefillParams& p, const PBars& bars,
                                                 volatile int* s_unit, int u, int uit,
                                                 volatile int* abort_flag, int lane) {
  if (p.sched == nullptr) return u + static_cast<int>(gridDim.x);
  int nxt = 0;
  if (lane == 0) {
    nxt = static_cast<int>(gridDim.x) + atomicAdd(p.sched, 1);
    const int k = (uit + 1) & 1, m = uit >> 1;
    if (pwait(bars.unit_empty + k, static_cast<uint32_t>((m & 1) ^ 1), abort_flag, p.status)) {
      s_unit[k] = nxt;
      mbar_arrive(bars.unit_full + k);  // release: the id is visible with the phase
    } else {
      nxt = INT_MAX;
    }
  }
  return __shfl_sync(0xffffffffu, nxt, 0);
}

// Next unit for a consumer (all lanes of a softmax warp, or the MMA thread
// alone: `single`).  INT_MAX after an abort.
__device__ __forceinline__ int next_unit(const PrefillParams& p, const PBars& bars,
                                         volatile int* s_unit, int u, int uit,
                                         volatile int* abort_flag, bool single, int lane) {
  if (p.sched == nullptr) return u + static_cast<int>(gridDim.x);
  const int k = (uit + 1) & 1, m = uit >> 1;
  if (!pwait(bars.unit_full + k, static_cast<uint32_t>(m & 1), abort_flag, p.status)) return INT_MAX;
  const int nxt = s_unit[k];
  if (!single) __syncwarp();
  if (single || lane == 0) mbar_arrive(bars.unit_empty + k);
  return nxt;
}

template <bool kBF16>
__global__ void __launch_bounds__(kThreads, 1)
    chunked_prefill_kernel(const __grid_constant__ PrefillParams p,
                           const __grid_constant__ CUtensorMap qmap,
                           const __grid_constant__ CUtensorMap kmap,
                           const __grid_constant__ CUtensorMap vmap) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  using L = PrefillSmem;
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + L::bar_off);
  PBars bars;
  bars.q_full = bar + 0;
  bars.q_empty = bar + 1;
  bars.kfull = bar + 2;
  bars.vfull = bar + 2 + kKvStages;
  bars.kempty = bar + 2 + 2 * kKvStages;
  bars.vempty = bar + 2 + 3 * kKvStages;
  bars.s_full = bar + 2 + 4 * kKvStages;
  bars.p_full = bar + 4 + 4 * kKvStages;
  bars.pv_done = bar + 6 + 4 * kKvStages;
  bars.unit_full = bar + 8 + 4 * kKvStages;
  bars.unit_empty = bar + 10 + 4 * kKvStages;
  bars.mx_full = bar + 12 + 4 * kKvStages;
  bars.ep_full = bar + 14 + 4 * kKvStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::misc_off);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::misc_off + 4);
  volatile int* s_unit = reinterpret_cast<volatile int*>(smem + L::misc_off + 8);
  int* prefix = reinterpret_cast<int*>(smem + L::table_off);
  float* s_mx = reinterpret_cast<float*>(smem + L::xchg_off);
  float* s_l = s_mx + 2 * 2 * 128;
  __shared__ int s_warp_tot[kThreads / 32];

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int B = p.num_seqs;
  const int G = p.group;
  const int tpt = p.tokens_per_tile;

  asm volatile("griddepcontrol.wait;" ::: "memory");
  // ---- prologue: M-tile pairs per sequence, exclusive prefix -------------------
  const int per = (B + blockDim.x - 1) / blockDim.x;
  const int b_lo = min(B, tid * per), b_hi = min(B, b_lo + per);
  auto pairs_of = [&](int b) {
    const int qlen = __ldg(p.qsl + b + 1) - __ldg(p.qsl + b);
    const int mt = qlen > 0 ? (qlen + tpt - 1) / tpt : 0;
    return (mt + 1) / 2;
  };
  int local = 0;
  for (int b = b_lo; b < b_hi; ++b) local += pairs_of(b);
  int incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) s_warp_tot[warp] = incl;
  if (tid == 0) {
    *abort_flag = 0;
    mbar_init(bars.q_full, 1);
    mbar_init(bars.q_empty, 1);
    for (int s = 0; s < kKvStages; ++s) {
      mbar_init(bars.kfull + s, 1);
      mbar_init(bars.vfull + s, 1);
      mbar_init(bars.kempty + s, 1);
      mbar_init(bars.vempty + s, 1);
    }
    for (int x = 0; x < 2; ++x) {
      mbar_init(bars.s_full + x, 1);
      mbar_init(bars.p_full + x, 8);
      mbar_init(bars.mx_full + x, 8);
      mbar_init(bars.pv_done + x, 1);
      mbar_init(bars.unit_full + x, 1);
      mbar_init(bars.unit_empty + x, kUnitConsumers);
    }
    mbar_init(bars.ep_full, 8);
    fence_mbar_init();
    tma_prefetch_desc(&qmap);
    tma_prefetch_desc(&kmap);
    tma_prefetch_desc(&vmap);
  }
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, 512);
    tc::tmem_relinquish();
  }
  __syncthreads();
  {
    int warp_off = 0;
    for (int w = 0; w < warp; ++w) warp_off += s_warp_tot[w];
    int run = warp_off + incl - local;
    for (int b = b_lo; b < b_hi; ++b) {
      prefix[b] = run;
      run += pairs_of(b);
    }
    if (tid == blockDim.x - 1) prefix[B] = warp_off + incl;
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  const int total_units = prefix[B] * p.num_kv_heads;

  uint8_t* sQ = smem + L::q_off;
  uint8_t* sK = smem + L::k_off;
  uint8_t* sV = smem + L::v_off;
  const int spb = p.block_size / 16;

  if (warp == 0) {
    // =========================== TMA producer ===========================
    // Warp-wide: block-table entries are fetched 32 at a time into a register
    // and handed out by shuffle; lane i issues page i of a KV tile.
    int t = 0, uit = 0;
    int bt_b = -1, bt_e0 = 0, bt_reg = 0;
    for (int u = blockIdx.x; u < total_units && !*abort_flag; ++uit) {
      const UnitInfo ui = unit_info(p, prefix, u);
      if (!pwait(bars.q_empty, (uit & 1) ^ 1, abort_flag, p.status)) break;
      if (lane == 0) {
        // each box spans tpt tokens (rows past the sequence are the next
        // sequence's or zero fill) and TMA delivers the whole box
        mbar_arrive_expect_tx(bars.q_full, 2 * tpt * G * 2 * 128);
        for (int x = 0; x < 2; ++x) {
          const int tok = ui.qrow0 + ui.t0 + x * tpt;
          tma_load_3d(sQ + x * kTileBytes, &qmap, bars.q_full, 0, ui.h * G, tok);
          tma_load_3d(sQ + x * kTileBytes + kRegionBytes, &qmap, bars.q_full, 64, ui.h * G, tok);
        }
      }
      const int npages_needed = (ui.kv_end + 15) / 16;
      const int* bt = p.block_table + static_cast<int64_t>(ui.b) * p.bt_stride;
      bool ok = true;
      for (int j = 0; j < ui.ntiles; ++j, ++t) {
        const int s = t % kKvStages;
        const uint32_t n = static_cast<uint32_t>(t / kKvStages);
        const int pg0 = j * 8;
        const int npg = min(8, npages_needed - pg0);
        const int e_first = pg0 / spb, e_last = (pg0 + npg - 1) / spb;
        if (ui.b != bt_b || e_first < bt_e0 || e_last >= bt_e0 + 32) {
          bt_b = ui.b;
          bt_e0 = e_first;
          const int idx = e_first + lane;
          bt_reg = idx < p.max_blocks_per_seq ? __ldg(bt + idx) : -1;
        }
        const int pg = pg0 + (lane < npg ? lane : 0);
        int blk = __shfl_sync(0xffffffffu, bt_reg, pg / spb - bt_e0);
        if (lane < npg && (blk < 0 || blk >= p.num_blocks)) {
          set_status(p.status, PS_DEV_BLOCK_OUT_OF_RANGE);
          blk = 0;
        }
        const int tok = (pg % spb) * 16;
        const uint32_t bytes = static_cast<uint32_t>(npg) * 2 * 2048;
        // K as soon as both S products of the stage's previous K tile are
        // done, V once both PV products of its previous V tile are: the K
        // tile (needed first) starts loading a PV pair earlier
        if (!pwait(bars.kempty + s, (n & 1) ^ 1, abort_flag, p.status)) { ok = false; break; }
        uint8_t* kd = sK + s * kTileBytes;
        if (lane == 0) mbar_arrive_expect_tx(bars.kfull + s, bytes);
        __syncwarp();  // armed before any copy completes
        if (lane < npg) {
          tma_load_4d(kd + lane * 2048, &kmap, bars.kfull + s, 0, ui.h, tok, blk);
          tma_load_4d(kd + kRegionBytes + lane * 2048, &kmap, bars.kfull + s, 64, ui.h, tok, blk);
        }
        if (!pwait(bars.vempty + s, (n & 1) ^ 1, abort_flag, p.status)) { ok = false; break; }
        uint8_t* vd = sV + s * kTileBytes;
        if (lane == 0) mbar_arrive_expect_tx(bars.vfull + s, bytes);
        __syncwarp();
        if (lane < npg) {
          tma_load_4d(vd + lane * 2048, &vmap, bars.vfull + s, 0, ui.h, tok, blk);
          tma_load_4d(vd + kRegionBytes + lane * 2048, &vmap, bars.vfull + s, 64, ui.h, tok, blk);
        }
      }
      if (!ok) break;
      u = claim_and_publish(p, bars, s_unit, u, uit, abort_flag, lane);
    }
  } else if (warp == 1) {
    // =========================== MMA issuer ===========================
    if (lane == 0) {
      const uint32_t idesc_qk = tc::idesc_f16(kBF16, 128, 128, false, false);
      const uint32_t idesc_pv = tc::idesc_f16(kBF16, 128, 128, false, true);
      const uint32_t q_addr = smem_u32(sQ), k_addr = smem_u32(sK), v_addr = smem_u32(sV);
      auto issue_s = [&](int x, int s) {
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off = (kk >> 2) * kRegionBytes + (kk & 3) * 32;
          const uint64_t ad = tc::sw128_desc(q_addr + x * kTileBytes + off, 16, 1024);
          const uint64_t bd = tc::sw128_desc(k_addr + s * kTileBytes + off, 16, 1024);
          tc::mma_f16_ss(tmem + x * 128, ad, bd, idesc_qk, kk > 0 ? 1u : 0u);
        }
        tc::commit(bars.s_full + x);
      };
      // PV of tile x for global KV tile tt; P sits in S_x's first 64 columns as
      // packed 16-bit pairs (keys 16kk.. = columns 8kk..)
      auto issue_pv = [&](int x, int tt, int jj) -> bool {
        const int s = tt % kKvStages;
        if (!pwait(bars.p_full + x, static_cast<uint32_t>(tt & 1), abort_flag, p.status)) return false;
        if (x == 0 &&
            !pwait(bars.vfull + s, static_cast<uint32_t>((tt / kKvStages) & 1), abort_flag, p.status))
          return false;
        tc::fence_after_sync();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t bd = tc::sw128_desc(v_addr + s * kTileBytes + kk * 2048, kRegionBytes, 1024);
          tc::mma_f16_ts(tmem + 256 + x * 128, tmem + x * 128 + kk * 8, bd, idesc_pv,
                         (jj > 0 || kk > 0) ? 1u : 0u);
        }
        tc::commit(bars.pv_done + x);
        if (x == 1) tc::commit(bars.vempty + s);  // both PVs of this stage issued
        return true;
      };
      int t = 0, uit = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < total_units && ok; ++uit) {
        const UnitInfo ui = unit_info(p, prefix, u);
        if (!pwait(bars.q_full, static_cast<uint32_t>(uit & 1), abort_flag, p.status)) break;
        tc::fence_after_sync();
        {  // S_A(0), S_B(0)
          const int s = t % kKvStages;
          if (!pwait(bars.kfull + s, static_cast<uint32_t>((t / kKvStages) & 1), abort_flag, p.status)) break;
          tc::fence_after_sync();
          issue_s(0, s);
          issue_s(1, s);
          tc::commit(bars.kempty + s);
          if (ui.ntiles == 1) tc::commit(bars.q_empty);
        }
        for (int j = 0; j < ui.ntiles; ++j) {
          const int tt = t + j;
          const bool more = j + 1 < ui.ntiles;
          const int sn = (tt + 1) % kKvStages;
          if (!issue_pv(0, tt, j)) { ok = false; break; }
          if (more) {
            if (!pwait(bars.kfull + sn, static_cast<uint32_t>(((tt + 1) / kKvStages) & 1), abort_flag,
                       p.status)) { ok = false; break; }
            tc::fence_after_sync();
            issue_s(0, sn);  // S_A(j+1) after PV_A(j): same TMEM columns, issue order
          }
          if (!issue_pv(1, tt, j)) { ok = false; break; }
          if (more) {
            issue_s(1, sn);
            tc::commit(bars.kempty + sn);
            if (j + 1 == ui.ntiles - 1) tc::commit(bars.q_empty);
          }
        }
        t += ui.ntiles;
        if (ok) u = next_unit(p, bars, s_unit, u, uit, abort_flag, true, lane);
      }
    }
  } else if (warp >= 4) {
    // =========================== softmax + epilogue ===========================
    // Both warpgroups work on every tile, A then B: warpgroup h (warps 4-7:
    // h = 0, warps 8-11: h = 1) takes keys [64h, 64h + 64) of each row (one
    // thread per TMEM lane = M row), so a tile's softmax is spread over 256
    // threads.  The two halves of a row agree on its max through shared
    // memory (mx_bar) before exponentiating, and on its sum at the epilogue.
    const int half = (warp >= 8) ? 1 : 0;
    const int quarter = warp & 3;             // TMEM lane quarter this warp may access
    const int row = quarter * 32 + lane;      // M row == TMEM lane
    const int ctid = half * 128 + row;        // 0..255 over the two warpgroups
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    // per-tensor cache scales fold into the score scale (K) and the output
    // normalisation (V)
    const float sl2 = p.scale_log2 * (p.k_scale ? __ldg(p.k_scale) : 1.f);
    const float v_scale = p.v_scale ? __ldg(p.v_scale) : 1.f;
    int t = 0, uit = 0;
    for (int u = blockIdx.x; u < total_units; ++uit) {
      const UnitInfo ui = unit_info(p, prefix, u);
      int tok[2], limit[2];
      bool row_valid[2];
      float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
#pragma unroll
      for (int x = 0; x < 2; ++x) {
        tok[x] = ui.t0 + x * tpt + row / G;
        row_valid[x] = row < tpt * G && tok[x] < ui.qlen;
        limit[x] = row_valid[x] ? ui.ctx + tok[x] : -1;  // last visible key
      }
      const int hin = row - (row / G) * G;
      bool ok = true;
      for (int j = 0; j < ui.ntiles && ok; ++j, ++t) {
#pragma unroll
        for (int x = 0; x < 2; ++x) {
          const uint32_t s_addr = lane_addr + x * 128;
          if (!pwait(bars.s_full + x, static_cast<uint32_t>(t & 1), abort_flag, p.status)) { ok = false; break; }
          tc::fence_after_sync();
          const int key0 = j * kKeys + 64 * half;
          const bool need_mask = !__all_sync(0xffffffffu, key0 + 63 <= limit[x]);
          // this half's 64 raw scores, one TMEM round trip
          uint32_t r[2][32];
          tc::ld_32x32b_x32(s_addr + 64 * half, r[0]);
          tc::ld_32x32b_x32(s_addr + 64 * half + 32, r[1]);
          tc::wait_ld();
          if (need_mask) {
#pragma unroll
            for (int c = 0; c < 2; ++c)
#pragma unroll
              for (int i = 0; i < 32; ++i)
                if (key0 + 32 * c + i > limit[x]) r[c][i] = __float_as_uint(-INFINITY);
          }
          float mxp[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) mxp[i] = -INFINITY;
#pragma unroll
          for (int c = 0; c < 2; ++c)
#pragma unroll
            for (int i = 0; i < 16; ++i)
              mxp[i & 7] = max3(mxp[i & 7], __uint_as_float(r[c][2 * i]), __uint_as_float(r[c][2 * i + 1]));
          const float mx_own =
              fmaxf(max3(mxp[0], mxp[1], mxp[2]), max3(mxp[3], mxp[4], max3(mxp[5], mxp[6], mxp[7])));
          // exchange with the other half of the row (every S read of this tile
          // precedes the arrive, so P may then overwrite any S column)
          s_mx[(x * 2 + half) * 128 + row] = mx_own;
          tc::fence_before_sync();
          __syncwarp();
          if (lane == 0) mbar_arrive(bars.mx_full + x);
          if (!pwait(bars.mx_full + x, static_cast<uint32_t>(t & 1), abort_flag, p.status)) { ok = false; break; }
          tc::fence_after_sync();
          float mx = fmaxf(mx_own, s_mx[(x * 2 + (half ^ 1)) * 128 + row]);
          mx *= sl2;  // scale > 0: max of scaled = scaled max
          float m_new = m_run[x], factor = 1.f;
          if (mx > m_run[x] + kRescaleThreshold || (m_run[x] == -INFINITY && mx > -INFINITY)) {
            m_new = mx;
            factor = ex2(m_run[x] - m_new);  // 0 when m_run == -inf
          }
          const float neg_m = (m_new == -INFINITY) ? 0.f : -m_new;  // fully masked row: all p = 0
          // O lives in TMEM: rescaling it needs the previous PV of this tile
          // done; each half rescales its 64 output dims
          if (j > 0 && __any_sync(0xffffffffu, factor != 1.f)) {
            if (!pwait(bars.pv_done + x, static_cast<uint32_t>((t - 1) & 1), abort_flag, p.status)) {
              ok = false;
              break;
            }
            tc::fence_after_sync();
            const uint32_t o_addr = lane_addr + 256 + x * 128 + 64 * half;
#pragma unroll
            for (int c = 0; c < 2; ++c) {
              uint32_t o[32];
              tc::ld_32x32b_x32(o_addr + c * 32, o);
              tc::wait_ld();
#pragma unroll
              for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * factor);
              tc::st_32x32b_x32(o_addr + c * 32, o);
            }
          }
          // p = exp2(s * scale - m), packed to 16 bit into P columns
          // [32h, 32h + 32) (keys 64h .. 64h + 63); pairs of elements go
          // through the packed f32x2 FMA and add
          uint64_t rsp[4] = {0ull, 0ull, 0ull, 0ull};
          const uint64_t sl2x2 = f2_pack(sl2, sl2), negm_x2 = f2_pack(neg_m, neg_m);
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            uint32_t pk[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              float x0, x1;
              f2_unpack(f2_fma(f2_pack(__uint_as_float(r[c][2 * i]), __uint_as_float(r[c][2 * i + 1])), sl2x2,
                               negm_x2),
                        x0, x1);
              const float p0 = ((2 * i) % 8 < PS_PREFILL_EMU_PER8) ? exp2_fma(x0) : ex2(x0);
              const float p1 = ((2 * i + 1) % 8 < PS_PREFILL_EMU_PER8) ? exp2_fma(x1) : ex2(x1);
              rsp[i & 3] = f2_add(rsp[i & 3], f2_pack(p0, p1));
              pk[i] = pack2<kBF16>(p0, p1);
            }
            tmem_st_x16(s_addr + 32 * half + 16 * c, pk);
          }
          float rs;
          {
            float a0, a1, b0, b1;
            f2_unpack(f2_add(rsp[0], rsp[1]), a0, a1);
            f2_unpack(f2_add(rsp[2], rsp[3]), b0, b1);
            rs = (a0 + b0) + (a1 + b1);
          }
          l_run[x] = l_run[x] * factor + rs;  // this half's keys; both halves apply the same factors
          m_run[x] = m_new;
          tc::wait_st();
          // last tile of the unit: V rows at or past kv_end must be finite
          // (zero) before PV_A reads them (PV_B is issued after PV_A)
          if (x == 0 && j == ui.ntiles - 1) {
            const int z0 = ui.kv_end - j * kKeys;
            if (z0 < kKeys) {
              const int s = t % kKvStages;
              if (!pwait(bars.vfull + s, static_cast<uint32_t>((t / kKvStages) & 1), abort_flag, p.status)) {
                ok = false;
                break;
              }
              uint8_t* vd = sV + s * kTileBytes;
              const int nchunks = (kKeys - z0) * 16;  // 16-byte chunks over both regions
              for (int i = ctid; i < nchunks; i += 256) {
                const int rr = z0 + (i >> 4);
                const int region = (i >> 3) & 1;
                *reinterpret_cast<uint4*>(vd + region * kRegionBytes + rr * 128 + (i & 7) * 16) =
                    make_uint4(0u, 0u, 0u, 0u);
              }
              fence_proxy_async_smem();  // generic writes before the tensor core reads V
            }
          }
          tc::fence_before_sync();
          __syncwarp();
          if (lane == 0) mbar_arrive(bars.p_full + x);
        }
      }
      if (!ok) break;
      // ---- epilogue: O / l -> global; each half writes its 64 dims ----
      bool done_ok = true;
#pragma unroll
      for (int x = 0; x < 2; ++x) {
        if (!pwait(bars.pv_done + x, static_cast<uint32_t>((t - 1) & 1), abort_flag, p.status)) done_ok = false;
        s_l[(x * 2 + half) * 128 + row] = l_run[x];
      }
      if (!done_ok) break;
      tc::fence_after_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(bars.ep_full);
      if (!pwait(bars.ep_full, static_cast<uint32_t>(uit & 1), abort_flag, p.status)) break;
#pragma unroll
      for (int x = 0; x < 2; ++x) {
        const float l_tot = l_run[x] + s_l[(x * 2 + (half ^ 1)) * 128 + row];
        const bool zero = (l_tot == 0.f) || (l_tot != l_tot);
        const float inv = zero ? 0.f : v_scale / l_tot;
        const int qh = ui.h * G + hin;
        const int64_t orow = static_cast<int64_t>(ui.qrow0 + tok[x]);
        const uint32_t o_addr = lane_addr + 256 + x * 128 + 64 * half;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t o[32];
          tc::ld_32x32b_x32(o_addr + c * 32, o);
          tc::wait_ld();
          if (row_valid[x]) {
            uint8_t* dst = reinterpret_cast<uint8_t*>(p.out) +
                           (orow * p.o_st + static_cast<int64_t>(qh) * p.o_sh + 64 * half + c * 32) * 2;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              uint4 v;
              v.x = pack2<kBF16>(__uint_as_float(o[8 * i + 0]) * inv, __uint_as_float(o[8 * i + 1]) * inv);
              v.y = pack2<kBF16>(__uint_as_float(o[8 * i + 2]) * inv, __uint_as_float(o[8 * i + 3]) * inv);
              v.z = pack2<kBF16>(__uint_as_float(o[8 * i + 4]) * inv, __uint_as_float(o[8 * i + 5]) * inv);
              v.w = pack2<kBF16>(__uint_as_float(o[8 * i + 6]) * inv, __uint_as_float(o[8 * i + 7]) * inv);
              *reinterpret_cast<uint4*>(dst + i * 16) = v;
            }
          }
        }
        if (half == 0 && row_valid[x] && p.lse != nullptr)
          p.lse[static_cast<int64_t>(qh) * p.lse_sh + orow * p.lse_st] =
              zero ? -INFINITY : (m_run[x] + __log2f(l_tot)) * 0.6931471805599453f;
      }
      tc::fence_before_sync();
      u = next_unit(p, bars, s_unit, u, uit, abort_flag, false, lane);
    }
  }
  // ---- teardown: every role done; TMEM owner frees it ----
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if (warp == 1) tc::tmem_dealloc(tmem, 512);
  // the last CTA out resets the scheduler (every CTA made its last claim
  // before its threads met above)
  if (tid == 0 && p.sched != nullptr) {
    __threadfence();
    if (atomicAdd(p.sched + 1, 1) == static_cast<int>(gridDim.x) - 1) {
      p.sched[0] = 0;
      p.sched[1] = 0;
    }
  }
}

template <bool kBF16>
static int launch_prefill_t(const PrefillParams& p, const CUtensorMap& qmap, const CUtensorMap& kmap,
                            const CUtensorMap& vmap, int grid, cudaStream_t stream) {
  const size_t smem = 1024 + PrefillSmem::bytes_before_table + static_cast<size_t>(p.num_seqs + 1) * 4;
  static bool configured[64] = {false};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev >= 64) return static_cast<int>(cudaErrorInvalidDevice);
  if (!configured[dev]) {
    const cudaError_t e = cudaFuncSetAttribute(
        chunked_prefill_kernel<kBF16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
        static_cast<int>(1024 + PrefillSmem::bytes_before_table + (kPrefillMaxSeqs + 1) * 4));
    if (e != cudaSuccess) return static_cast<int>(e);
    configured[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, chunked_prefill_kernel<kBF16>, p, qmap, kmap, vmap);
  return static_cast<int>(e != cudaSuccess ? e : cudaGetLastError());
}

}  // namespace ps

int ps_launch_chunked_prefill(const ps::PrefillParams& p, const CUtensorMap& qmap,
                              const CUtensorMap& kmap, const CUtensorMap& vmap, int dtype_bf16,
                              int grid, cudaStream_t stream) {
  return dtype_bf16 ? ps::launch_prefill_t<true>(p, qmap, kmap, vmap, grid, stream)
                    : ps::launch_prefill_t<false>(p, qmap, kmap, vmap, grid, stream);
}
