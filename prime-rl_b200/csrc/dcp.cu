// Decode context parallelism (DCP) over NVLink peer memory.
//
// The N ranks of a DCP group hold interleaved slices of every sequence's KV
// tokens: position p lives on rank (p / I) % N (I = interleave), at local
// index (p / (N*I)) * I + p % I of that rank's paged cache, with the block
// table shared by all ranks (vllm/v1/worker/block_table.py:357-376).  Each
// rank holds hq_local query heads; the group's query heads are the
// concatenation over ranks (rank r: heads [r*hq_local, (r+1)*hq_local)).
//
// One DCP decode call per rank replaces vLLM's FlashAttentionImpl
// ._forward_with_dcp (vllm/v1/attention/backends/flash_attn.py:885-983):
//   query all_gather over the group          -> dcp_stage_kernel + dcp_gather_kernel
//   attention over the local context (FA)     -> paged_decode_kernel (unchanged)
//   cp_lse_ag_out_rs: LSE all_gather, correct_attn_out, reduce_scatter
//   (vllm/v1/attention/ops/common.py:99-225)  -> dcp_combine_kernel
//   attention of the new token over itself + merge_attn_states
//   (merge_attn_states.py:9, triton_merge_attn_states.py:58-140)
//                                             -> dcp_combine_kernel
//   reshape_and_cache_flash of the new token  -> dcp_combine_kernel
// The exchanges are loads of the peers' slabs (IPC-mapped device memory) and
// no NCCL call is made.  Two flag barriers per call: phase 0 (every rank's
// query rows staged) and phase 1 (every rank's partial outputs written).
// Each protects the buffer the other phase's readers use, so no barrier is
// needed at the end of a call: a rank restages its query rows only after all
// ranks entered phase 1 of the previous call (so they finished reading them),
// and rewrites its partials only after all ranks entered phase 0 of the next
// call.
//
// Slab layout (identical on every rank, offsets from dcp_layout):
//   [0, 256)    the synchronisation header of peer_sync.cuh
//   off_q       [max_tokens, hq_local, 128] query rows staged for the peers
//   off_part    [max_tokens, hq_all, 128] partial outputs over the local context
//   off_lse     [hq_all, max_tokens] fp32 partial LSEs (natural log)
//   off_qall    [max_tokens, hq_all, 128] the group's query rows (local)
//   off_lens    [max_tokens] int32 local context lengths (local)
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "peer_sync.cuh"
#include "ps_common.cuh"
#include "ps_launch.h"

namespace ps {
namespace {

__device__ __forceinline__ int32_t call_epoch(const DcpArgs& a) { return peer::call_epoch(a.slab[a.rank]); }

__device__ __forceinline__ void signal_phase(const DcpArgs& a, int ph, int32_t e) {
  peer::signal(a.slab, a.world, a.rank, ph, e);
}

// false after a timeout: the caller skips the phase's reads of peer data
__device__ __forceinline__ bool wait_phase(const DcpArgs& a, int ph, int32_t e) {
  return peer::wait_all(a.slab[a.rank], a.world, ph, e, a.status);
}

__device__ __forceinline__ uint4 ld16(const char* p) { return *reinterpret_cast<const uint4*>(p); }
__device__ __forceinline__ void st16(char* p, uint4 v) { *reinterpret_cast<uint4*>(p) = v; }

}  // namespace

// Stage this rank's query rows into its slab for the peers, and compute the
// local context length of every sequence: the count of positions
// p < seq_len - 1 (the new token excluded) with (p / I) % N == rank, as
// vllm/v1/attention/backends/utils.py:857-894 (get_dcp_local_seq_lens) does.
__global__ void __launch_bounds__(256) dcp_stage_kernel(const __grid_constant__ DcpArgs a) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  char* own = a.slab[a.rank];
  const int64_t gtid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t gstride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t nvec = static_cast<int64_t>(a.num_tokens) * a.hq_local * 16;
  for (int64_t i = gtid; i < nvec; i += gstride) {
    const int64_t row = i >> 4;
    const int c = static_cast<int>(i & 15);
    const int64_t t = row / a.hq_local;
    const int64_t h = row - t * a.hq_local;
    st16(own + a.off_q + row * 256 + c * 16, ld16(a.q + t * a.q_st + h * a.q_sh + c * 16));
  }
  int32_t* lens = reinterpret_cast<int32_t*>(own + a.off_lens);
  const int64_t span = static_cast<int64_t>(a.world) * a.interleave;
  for (int64_t b = gtid; b < a.num_tokens; b += gstride) {
    int64_t ctx = static_cast<int64_t>(a.seq_lens[b]) - 1;
    if (ctx < 0) {
      set_status(a.status, PS_DEV_BAD_METADATA);
      ctx = 0;
    }
    const int64_t full = ctx / span;
    const int64_t rem = ctx - full * span - static_cast<int64_t>(a.rank) * a.interleave;
    lens[b] = static_cast<int32_t>(full * a.interleave + min(max(rem, int64_t(0)), int64_t(a.interleave)));
  }
}

// Publish phase `ph` of the current call to every rank (one CTA).  Used when
// one process drives every rank of a group in turn; otherwise the gather and
// combine kernels signal at their start.
__global__ void dcp_signal_kernel(const __grid_constant__ DcpArgs a, int ph) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  signal_phase(a, ph, call_epoch(a));
}

// After phase 0: copy the group's query rows [T, hq_all, 128] into this
// rank's slab (rank r's rows come from rank r's slab over NVLink), the
// all_gather(query, dim=1) of flash_attn.py:907.  Four 16-byte loads in
// flight per thread.
__global__ void __launch_bounds__(256) dcp_gather_kernel(const __grid_constant__ DcpArgs a) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int32_t e = call_epoch(a);
  if (a.signal_first && blockIdx.x == 0) signal_phase(a, 0, e);
  if (!wait_phase(a, 0, e)) return;
  char* own = a.slab[a.rank];
  const int64_t nvec = static_cast<int64_t>(a.num_tokens) * a.hq_all * 16;
  const int64_t gtid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t gstride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i0 = gtid; i0 < nvec; i0 += 4 * gstride) {
    uint4 v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int64_t i = i0 + u * gstride;
      if (i < nvec) {
        const int64_t row = i >> 4;
        const int c = static_cast<int>(i & 15);
        const int64_t t = row / a.hq_all;
        const int hg = static_cast<int>(row - t * a.hq_all);
        const int r = hg / a.hq_local;
        const int j = hg - r * a.hq_local;
        v[u] = ld16(a.slab[r] + a.off_q + (t * a.hq_local + j) * 256 + c * 16);
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int64_t i = i0 + u * gstride;
      if (i < nvec) st16(own + a.off_qall + i * 16, v[u]);
    }
  }
}

// After phase 1, one warp per (token, own query head) row: the group's
// partial outputs of the row are merged with their LSEs by
// correct_attn_out's rule (common.py:42-96: NaN and +inf LSEs count as -inf,
// a max of -inf counts as 0, factor_r = exp(lse_r - lse)) and summed (the
// reduce_scatter of common.py:218), then merged with the new token's
// attention over itself (output v, LSE scale * q.k) by merge_attn_states'
// rule.  All in fp32, rounded once to the output dtype.  Before waiting, the
// CTAs append the new tokens this rank stores (slot >= 0) to its cache.
template <bool kBF16>
__global__ void __launch_bounds__(256) dcp_combine_kernel(const __grid_constant__ DcpArgs a) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int32_t e = call_epoch(a);
  if (a.signal_first && blockIdx.x == 0) signal_phase(a, 1, e);
  const int64_t gtid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t gstride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  if (!a.context_only) {  // reshape_and_cache_flash of the tokens stored here
    const int64_t nvec = static_cast<int64_t>(a.num_tokens) * a.num_kv_heads * 16;
    for (int64_t i = gtid; i < nvec; i += gstride) {
      const int64_t row = i >> 4;
      const int c = static_cast<int>(i & 15);
      const int64_t t = row / a.num_kv_heads;
      const int64_t h = row - t * a.num_kv_heads;
      const int64_t slot = a.slot_mapping[t];
      if (slot < 0) continue;
      if (slot >= a.num_slots) {
        if (h == 0 && c == 0) set_status(a.status, PS_DEV_SLOT_OUT_OF_RANGE);
        continue;
      }
      const int64_t blk = slot / a.block_size;
      const int64_t dst = blk * a.c_sblock + (slot - blk * a.block_size) * a.c_sslot + h * a.c_shead + c * 16;
      st16(a.key_cache + dst, ld16(a.new_key + t * a.nk_st + h * a.nk_sh + c * 16));
      st16(a.value_cache + dst, ld16(a.new_value + t * a.nv_st + h * a.nv_sh + c * 16));
    }
  }
  if (wait_phase(a, 1, e)) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t rows = static_cast<int64_t>(a.num_tokens) * a.hq_local;
    const int world = a.world;
    for (int64_t row = static_cast<int64_t>(blockIdx.x) * 8 + warp; row < rows;
         row += static_cast<int64_t>(gridDim.x) * 8) {
      const int64_t t = row / a.hq_local;
      const int h = static_cast<int>(row - t * a.hq_local);
      const int hg = a.rank * a.hq_local + h;
      const int kvh = hg / a.group;
      // every load of the row first: LSEs (lane r: rank r), partial rows (4
      // elements per lane from each rank), the new token's q, k and v
      float l = -INFINITY;
      if (lane < world)
        l = reinterpret_cast<const float*>(a.slab[lane] + a.off_lse)[static_cast<int64_t>(hg) * a.num_tokens + t];
      uint2 pv[kDcpMaxWorld];
#pragma unroll
      for (int r = 0; r < kDcpMaxWorld; ++r)
        if (r < world)
          pv[r] = *reinterpret_cast<const uint2*>(a.slab[r] + a.off_part +
                                                  ((t * a.hq_all + hg) * 128 + lane * 4) * 2);
      uint2 qv = make_uint2(0u, 0u), kv = qv, vv = qv;
      if (!a.context_only) {
        qv = *reinterpret_cast<const uint2*>(a.q + t * a.q_st + h * a.q_sh + lane * 8);
        kv = *reinterpret_cast<const uint2*>(a.new_key + t * a.nk_st + kvh * a.nk_sh + lane * 8);
        vv = *reinterpret_cast<const uint2*>(a.new_value + t * a.nv_st + kvh * a.nv_sh + lane * 8);
      }
      // LSE over the ranks' partials
      if (l != l || l == INFINITY) l = -INFINITY;
      float mx = l;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      if (mx == -INFINITY) mx = 0.f;
      float se = lane < world ? __expf(l - mx) : 0.f;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) se += __shfl_xor_sync(0xffffffffu, se, o);
      const float lse_ctx = __logf(se) + mx;
      float f = l - lse_ctx;
      if (f != f || f == INFINITY) f = -INFINITY;
      f = __expf(f);
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int r = 0; r < kDcpMaxWorld; ++r) {
        if (r < world) {
          const float fr = __shfl_sync(0xffffffffu, f, r);
          const float2 x0 = unpack2<kBF16>(pv[r].x), x1 = unpack2<kBF16>(pv[r].y);
          acc[0] += fr * x0.x;
          acc[1] += fr * x0.y;
          acc[2] += fr * x1.x;
          acc[3] += fr * x1.y;
        }
      }
      if (a.context_only) {  // the corrected context attention, its LSE
        uint2 o;
        o.x = pack2<kBF16>(acc[0], acc[1]);
        o.y = pack2<kBF16>(acc[2], acc[3]);
        *reinterpret_cast<uint2*>(a.out + t * a.o_st + h * a.o_sh + lane * 8) = o;
        if (a.lse != nullptr && lane == 0) a.lse[h * a.lse_sh + t * a.lse_st] = lse_ctx;
        continue;
      }
      // the new token attending to itself
      const float2 q0 = unpack2<kBF16>(qv.x), q1 = unpack2<kBF16>(qv.y);
      const float2 k0 = unpack2<kBF16>(kv.x), k1 = unpack2<kBF16>(kv.y);
      float dot = q0.x * k0.x + q0.y * k0.y + q1.x * k1.x + q1.y * k1.y;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
      const float s = dot * a.softmax_scale;
      // merge_attn_states(context, new token)
      const float p = lse_ctx == INFINITY ? -INFINITY : lse_ctx;
      const float m2 = fmaxf(p, s);
      const float pse = __expf(p - m2), sse = __expf(s - m2);
      const float tot = pse + sse;
      const float wp = pse / tot, ws = sse / tot;
      const float2 v0 = unpack2<kBF16>(vv.x), v1 = unpack2<kBF16>(vv.y);
      uint2 o;
      o.x = pack2<kBF16>(acc[0] * wp + v0.x * ws, acc[1] * wp + v0.y * ws);
      o.y = pack2<kBF16>(acc[2] * wp + v1.x * ws, acc[3] * wp + v1.y * ws);
      *reinterpret_cast<uint2*>(a.out + t * a.o_st + h * a.o_sh + lane * 8) = o;
      if (a.lse != nullptr && lane == 0) a.lse[h * a.lse_sh + t * a.lse_st] = __logf(tot) + m2;
    }
  }
  // the last CTA out closes the call on this rank
  if (peer::last_cta(a.slab[a.rank])) peer::close_call(a.slab[a.rank], e);
}

}  // namespace ps

// which: 0 stage, 1 signal phase 0, 2 gather, 3 signal phase 1, 4 combine
int ps_launch_dcp(const ps::DcpArgs& a, int which, int sm_count, cudaStream_t stream) {
  auto grid_for = [&](int64_t units, int64_t per_cta, int64_t cap) {
    int64_t g = (units + per_cta - 1) / per_cta;
    if (g < 1) g = 1;
    if (g > cap) g = cap;
    return static_cast<unsigned>(g);
  };
  cudaLaunchConfig_t cfg = {};
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cfg.blockDim = dim3(256);
  // grids stay within one wave (2 CTAs of 256 threads per SM) so that every
  // CTA of a waiting kernel is resident and a timeout costs one wait
  const int64_t cap = 2LL * sm_count;
  cudaError_t e = cudaSuccess;
  switch (which) {
    case 0:
      cfg.gridDim = dim3(grid_for(static_cast<int64_t>(a.num_tokens) * a.hq_local * 16, 256, cap));
      e = cudaLaunchKernelEx(&cfg, ps::dcp_stage_kernel, a);
      break;
    case 1:
    case 3:
      cfg.gridDim = dim3(1);
      cfg.blockDim = dim3(32);
      e = cudaLaunchKernelEx(&cfg, ps::dcp_signal_kernel, a, which == 1 ? 0 : 1);
      break;
    case 2:
      cfg.gridDim = dim3(grid_for(static_cast<int64_t>(a.num_tokens) * a.hq_all * 16, 1024, cap));
      e = cudaLaunchKernelEx(&cfg, ps::dcp_gather_kernel, a);
      break;
    case 4:
      cfg.gridDim = dim3(grid_for(static_cast<int64_t>(a.num_tokens) * a.hq_local, 8, cap));
      e = a.bf16 ? cudaLaunchKernelEx(&cfg, ps::dcp_combine_kernel<true>, a)
                 : cudaLaunchKernelEx(&cfg, ps::dcp_combine_kernel<false>, a);
      break;
    default:
      return static_cast<int>(cudaErrorInvalidValue);
  }
  return static_cast<int>(e != cudaSuccess ? e : cudaGetLastError());
}

namespace ps {

// merge_attn_states: one warp per (token, head) row, 4 elements per lane.
template <bool kBF16>
__global__ void __launch_bounds__(256) merge_attn_states_kernel(const MergeArgs a) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t rows = a.num_tokens * a.num_heads;
  for (int64_t row = static_cast<int64_t>(blockIdx.x) * 8 + warp; row < rows;
       row += static_cast<int64_t>(gridDim.x) * 8) {
    const int64_t t = row / a.num_heads;
    const int h = static_cast<int>(row - t * a.num_heads);
    float p = a.p_lse[h * a.num_tokens + t];
    float s = a.s_lse[h * a.num_tokens + t];
    p = p == INFINITY ? -INFINITY : p;
    s = s == INFINITY ? -INFINITY : s;
    const float mx = fmaxf(p, s);
    const float pse = __expf(p - mx), sse = __expf(s - mx);
    const float tot = pse + sse;
    const float wp = pse / tot, ws = sse / tot;
    const uint2 pv = *reinterpret_cast<const uint2*>(a.p_out + t * a.p_st + h * a.p_sh + lane * 8);
    const uint2 sv = *reinterpret_cast<const uint2*>(a.s_out + t * a.s_st + h * a.s_sh + lane * 8);
    const float2 p0 = unpack2<kBF16>(pv.x), p1 = unpack2<kBF16>(pv.y);
    const float2 s0 = unpack2<kBF16>(sv.x), s1 = unpack2<kBF16>(sv.y);
    uint2 o;
    o.x = pack2<kBF16>(p0.x * wp + s0.x * ws, p0.y * wp + s0.y * ws);
    o.y = pack2<kBF16>(p1.x * wp + s1.x * ws, p1.y * wp + s1.y * ws);
    __syncwarp();  // out may alias an input: every lane has read its row
    *reinterpret_cast<uint2*>(a.out + t * a.o_st + h * a.o_sh + lane * 8) = o;
    if (a.out_lse != nullptr && lane == 0) a.out_lse[h * a.num_tokens + t] = __logf(tot) + mx;
  }
}

}  // namespace ps

int ps_launch_merge_attn_states(const ps::MergeArgs& a, int dtype_bf16, int sm_count,
                                cudaStream_t stream) {
  const int64_t rows = a.num_tokens * a.num_heads;
  if (rows == 0) return 0;
  int64_t g = (rows + 7) / 8;
  const int64_t cap = 8LL * sm_count;
  if (g > cap) g = cap;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(g));
  cfg.blockDim = dim3(256);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = dtype_bf16 ? cudaLaunchKernelEx(&cfg, ps::merge_attn_states_kernel<true>, a)
                                   : cudaLaunchKernelEx(&cfg, ps::merge_attn_states_kernel<false>, a);
  return static_cast<int>(e != cudaSuccess ? e : cudaGetLastError());
}
