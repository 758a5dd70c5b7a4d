// Head all-gather of a KV-head-sharded decode over NVLink peer memory.
//
// Each rank of the group attends with its own query heads (its KV heads'
// GQA groups) and the decode writes those rows, [T, hq_local, 128], into the
// rank's slab at kHeadGatherRowsOffset.  One launch per rank then replaces
// NCCL's all_gather_into_tensor plus the permute to [T, world * hq_local, 128]:
//   barrier 0 ("rows ready": every rank's decode completed),
//   every rank's rows pulled into `out` at head offset r * hq_local (16-byte
//   NVLink loads, four in flight per thread),
//   barrier 1 ("rows pulled"), waited by the grid's last CTA only, so that
//   no rank's next decode overwrites rows a peer is still reading.
// Slab header and barrier rules: peer_sync.cuh.
#include "peer_sync.cuh"
#include "ps_common.cuh"
#include "ps_launch.h"

namespace ps {

// mode 0: the whole step; 1: pull only (barrier 0 signalled by a separate
// launch, barrier 1 signalled but not waited for: one process playing every
// rank on one GPU runs head_gather_finish_kernel after every rank's pull)
__global__ void __launch_bounds__(256) head_gather_kernel(const __grid_constant__ HeadGatherArgs a) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  char* own = a.slab[a.rank];
  const int32_t e = peer::call_epoch(own);
  if (a.mode == 0 && blockIdx.x == 0) peer::signal(a.slab, a.world, a.rank, 0, e);
  if (peer::wait_all(own, a.world, 0, e, a.status)) {
    const int hq_all = a.world * a.hq_local;
    const int64_t nvec = static_cast<int64_t>(a.num_tokens) * hq_all * 16;
    const int64_t gtid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t gstride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t i0 = gtid; i0 < nvec; i0 += 4 * gstride) {
      uint4 v[4];
      int64_t dst[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int64_t i = i0 + u * gstride;
        dst[u] = -1;
        if (i < nvec) {
          const int64_t row = i >> 4;
          const int c = static_cast<int>(i & 15);
          const int64_t t = row / hq_all;
          const int hg = static_cast<int>(row - t * hq_all);
          const int r = hg / a.hq_local;
          const int j = hg - r * a.hq_local;
          v[u] = *reinterpret_cast<const uint4*>(a.slab[r] + kHeadGatherRowsOffset +
                                                 (t * a.hq_local + j) * 256 + c * 16);
          dst[u] = t * a.o_st + hg * a.o_sh + c * 16;
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (dst[u] >= 0) *reinterpret_cast<uint4*>(a.out + dst[u]) = v[u];
    }
  }
  if (peer::last_cta(own)) {  // every CTA of this rank has pulled
    peer::signal(a.slab, a.world, a.rank, 1, e);
    if (a.mode == 0) {
      peer::wait_all(own, a.world, 1, e, a.status);
      peer::close_call(own, e);
    }
  }
}

// Barrier 0 alone (one CTA), for the pull-only mode.
__global__ void head_gather_signal_kernel(const __grid_constant__ HeadGatherArgs a) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  peer::signal(a.slab, a.world, a.rank, 0, peer::call_epoch(a.slab[a.rank]));
}

// Barrier 1's wait and the end of the call (one CTA), for the pull-only mode.
__global__ void head_gather_finish_kernel(const __grid_constant__ HeadGatherArgs a) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  char* own = a.slab[a.rank];
  const int32_t e = peer::call_epoch(own);
  peer::wait_all(own, a.world, 1, e, a.status);
  peer::close_call(own, e);
}

}  // namespace ps

// which: 0 the whole step; 1 barrier 0's signal; 2 pull only; 3 finish
int ps_launch_head_gather(const ps::HeadGatherArgs& a, int which, int sm_count, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaSuccess;
  if (which == 1 || which == 3) {
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(32);
    e = which == 1 ? cudaLaunchKernelEx(&cfg, ps::head_gather_signal_kernel, a)
                   : cudaLaunchKernelEx(&cfg, ps::head_gather_finish_kernel, a);
  } else {
    ps::HeadGatherArgs b = a;
    b.mode = which == 0 ? 0 : 1;
    const int64_t units = static_cast<int64_t>(a.num_tokens) * a.world * a.hq_local * 16;
    int64_t g = (units + 1023) / 1024;
    // one wave (2 CTAs of 256 threads per SM): every waiting CTA is resident
    const int64_t cap = 2LL * sm_count;
    g = g < 1 ? 1 : (g > cap ? cap : g);
    cfg.gridDim = dim3(static_cast<unsigned>(g));
    cfg.blockDim = dim3(256);
    e = cudaLaunchKernelEx(&cfg, ps::head_gather_kernel, b);
  }
  return static_cast<int>(e != cudaSuccess ? e : cudaGetLastError());
}
