// Shared-prefix plan for the cascade decode: which adjacent decode sequences
// read the same leading KV pages.
//
// vLLM decides cascade attention for a whole batch from one common prefix
// (vllm/v1/attention/backends/flash_attn.py:1088-1130, use_cascade_attention)
// and prefix caching gives requests that share a prompt the same physical
// blocks, i.e. identical leading block-table entries.  GRPO rollouts (n
// samples per prompt, scheduled adjacently) share per-group prefixes instead,
// so the plan is built per group from the block table itself:
//
//   full(b)   = complete 16-token pages before the page of b's last token
//               ((seq_len - 1) / 16; 0 unless b is a decode row)
//   shared(b) = leading pages whose block-table entries equal b-1's, capped
//               at min(full(b), full(b-1)); shared(0) = 0
//   b starts a new group when b == 0, shared(b) < min_shared_pages, or
//   shared(b) < shared(b+1) (b shares more with its successor than with its
//   predecessor: a tighter group begins at b)
//   group pages = min of shared(b) over the group's members after the first
//
// Groups with at least two members are listed.  A shared page is complete in
// every member and no member's last page is shared, so the pages never change
// while the group decodes.
//
// One launch: a warp per sequence compares block-table rows 32 entries at a
// time; the last CTA to finish (arrival counter in the plan buffer) forms the
// groups with block scans.
#include "ps_common.cuh"
#include "ps_launch.h"

namespace ps {

constexpr int kPlanThreads = 256;
constexpr int kPlanHeader = 32;

__device__ __forceinline__ int full_pages(const PlanArgs& a, int b) {
  int qlen = 1;
  if (a.qsl) qlen = __ldg(a.qsl + b + 1) - __ldg(a.qsl + b);
  const int L = __ldg(a.seq_lens + b);
  if (qlen != 1 || L < 1) return 0;
  const int maxp = a.max_blocks_per_seq * (a.block_size / 16);
  return min((L - 1) / 16, maxp);
}

// Exclusive scan over kPlanThreads threads; contains __syncthreads.
__device__ __forceinline__ int plan_block_scan(int v, int* s_warp, int* total) {
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
  for (int w = 0; w < kPlanThreads / 32; ++w) {
    const int x = s_warp[w];
    if (w < warp) off += x;
    tot += x;
  }
  __syncthreads();
  *total = tot;
  return off + incl - v;
}

__global__ void __launch_bounds__(kPlanThreads) cascade_plan_kernel(const PlanArgs a) {
  const int B = a.num_seqs;
  const int Gm = max(1, B / 2);
  int32_t* plan = a.plan;
  int32_t* seq_group = plan + kPlanHeader;
  int32_t* g_first = seq_group + B;
  int32_t* g_size = g_first + Gm;
  int32_t* g_pages = g_size + Gm;
  int32_t* shared = g_pages + Gm;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int sub = a.block_size / 16;

  // ---- phase 1: shared(b), one warp per sequence ------------------------------
  const int b = blockIdx.x * (kPlanThreads / 32) + warp;
  if (b < B) {
    int s = 0;
    if (a.enabled && b > 0) {
      const int F = min(full_pages(a, b), full_pages(a, b - 1));
      const int E = (F + sub - 1) / sub;  // block entries covering F pages
      const int32_t* r0 = a.block_table + static_cast<int64_t>(b - 1) * a.bt_stride;
      const int32_t* r1 = a.block_table + static_cast<int64_t>(b) * a.bt_stride;
      int matched = E;
      for (int e0 = 0; e0 < E; e0 += 32) {
        const int e = e0 + lane;
        const bool differ = e < E && __ldg(r0 + e) != __ldg(r1 + e);
        const unsigned m = __ballot_sync(0xffffffffu, differ);
        if (m) {
          matched = e0 + __ffs(m) - 1;
          break;
        }
      }
      s = min(matched * sub, F);
    }
    if (lane == 0) shared[b] = s;
  }

  // ---- the last CTA to arrive forms the groups --------------------------------
  __shared__ int s_last;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(plan + 1, 1) == static_cast<int>(gridDim.x) - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();

  __shared__ int s_warp[kPlanThreads / 32];
  extern __shared__ int sm[];  // gsize[B], gpages[B], gfirst[B], glist[B]
  int* gsize = sm;
  int* gpages = gsize + B;
  int* gfirst = gpages + B;
  int* glist = gfirst + B;

  const int per = (B + kPlanThreads - 1) / kPlanThreads;
  const int lo = min(B, static_cast<int>(threadIdx.x) * per), hi = min(B, lo + per);
  auto sh = [&](int i) { return __ldcg(shared + i); };
  auto is_start = [&](int i) {
    if (i == 0) return true;
    const int si = sh(i);
    return si < a.min_shared_pages || (i + 1 < B && si < sh(i + 1));
  };
  int nb = 0;
  for (int i = lo; i < hi; ++i) nb += is_start(i);
  int ngroups;
  const int gbase = plan_block_scan(nb, s_warp, &ngroups);
  for (int g = threadIdx.x; g < ngroups; g += kPlanThreads) {
    gsize[g] = 0;
    gpages[g] = 0x7fffffff;
  }
  __syncthreads();
  int gid = gbase - 1;
  for (int i = lo; i < hi; ++i) {
    if (is_start(i)) {
      ++gid;
      gfirst[gid] = i;
    } else {
      atomicMin(gpages + gid, sh(i));
    }
    atomicAdd(gsize + gid, 1);
  }
  __syncthreads();
  // list the groups with two or more members
  const int gper = (ngroups + kPlanThreads - 1) / kPlanThreads;
  const int glo = min(ngroups, static_cast<int>(threadIdx.x) * gper), ghi = min(ngroups, glo + gper);
  int nk = 0;
  for (int g = glo; g < ghi; ++g) nk += gsize[g] >= 2;
  int nlisted;
  int li = plan_block_scan(nk, s_warp, &nlisted);
  for (int g = glo; g < ghi; ++g) {
    if (gsize[g] >= 2) {
      g_first[li] = gfirst[g];
      g_size[li] = gsize[g];
      g_pages[li] = gpages[g];
      glist[g] = li++;
    } else {
      glist[g] = -1;
    }
  }
  __syncthreads();
  gid = gbase - 1;
  for (int i = lo; i < hi; ++i) {
    if (is_start(i)) ++gid;
    seq_group[i] = glist[gid];
  }
  if (threadIdx.x == 0) {
    plan[0] = nlisted;
    plan[1] = 0;  // arrival counter back to zero for the next build
  }
}

}  // namespace ps

int64_t ps_cascade_plan_words(int num_seqs) {
  const int64_t gm = num_seqs / 2 > 1 ? num_seqs / 2 : 1;
  return ps::kPlanHeader + 2 * static_cast<int64_t>(num_seqs) + 3 * gm;
}

int ps_launch_cascade_plan(const ps::PlanArgs& a, cudaStream_t stream) {
  const int B = a.num_seqs;
  const int warps = ps::kPlanThreads / 32;
  const int grid = (B + warps - 1) / warps;
  const size_t smem = static_cast<size_t>(4) * B * sizeof(int);
  static bool configured[64] = {false};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev >= 64) return static_cast<int>(cudaErrorInvalidDevice);
  if (!configured[dev]) {
    const cudaError_t e = cudaFuncSetAttribute(ps::cascade_plan_kernel,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               4 * ps::kCascadeMaxSeqs * static_cast<int>(sizeof(int)));
    if (e != cudaSuccess) return static_cast<int>(e);
    configured[dev] = true;
  }
  ps::cascade_plan_kernel<<<grid, ps::kPlanThreads, smem, stream>>>(a);
  return static_cast<int>(cudaGetLastError());
}
