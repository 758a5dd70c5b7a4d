// Flag barriers between the GPUs of a group over peer memory (NVLink).
//
// Every rank owns a "slab" of device memory that the others map with CUDA
// IPC.  Its first 256 bytes are the synchronisation header:
//   int32 words [0, 16)  flags[ph][r] (ph < 2, r < 8): the last call epoch
//                        rank r signalled for phase ph (written by rank r,
//                        remotely, st.release.sys)
//   int32 word 32        epoch: calls completed on this rank (local)
//   int32 word 33        done: CTAs of the current kernel that finished (local)
//   int32 word 34        done, second round (a kernel that counts arrivals twice)
// A call's epoch is one more than the calls completed, so every kernel of a
// call agrees on it without host state (CUDA graphs replay the same
// launches).  Waits are bounded (1 s of %globaltimer) and report
// PS_DEV_WAIT_TIMEOUT in the caller's status word instead of hanging; a CTA
// that finds the bit already set gives up at once.
#pragma once

#include "ps_common.cuh"

namespace ps {
namespace peer {

constexpr int kEpochWord = 32;
constexpr int kDoneWord = 33;
constexpr long long kWaitNs = 1000000000LL;  // 1 s per barrier wait

__device__ __forceinline__ int32_t* words(char* slab) { return reinterpret_cast<int32_t*>(slab); }

__device__ __forceinline__ long long global_ns() {
  long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void store_release_sys(int32_t* p, int32_t v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ int32_t load_acquire_sys(const int32_t* p) {
  int32_t v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ int32_t load_volatile(const int32_t* p) {
  return *reinterpret_cast<const volatile int32_t*>(p);
}

// The epoch of the call in progress on the rank that owns `own`.
__device__ __forceinline__ int32_t call_epoch(char* own) {
  return load_volatile(words(own) + kEpochWord) + 1;
}

// Threads [0, world) of one CTA: publish "phase ph of call e done on `rank`"
// into every rank's flag array (own included).  The data the phase covers
// was written by earlier kernels of the stream, complete once
// griddepcontrol.wait returned, or by this CTA before a __syncthreads.
__device__ __forceinline__ void signal(char* const* slabs, int world, int rank, int ph, int32_t e) {
  const int r = threadIdx.x;
  if (r < world) {
    __threadfence_system();
    store_release_sys(words(slabs[r]) + ph * 8 + rank, e);
  }
}

// CTA-wide: whether every rank signalled phase ph of call e.  Threads
// [0, world) poll one flag each.  Contains __syncthreads.
__device__ __forceinline__ bool wait_all(char* own, int world, int ph, int32_t e, int32_t* status) {
  __shared__ int s_ok;
  if (threadIdx.x == 0) s_ok = 1;
  __syncthreads();
  const int r = threadIdx.x;
  if (r < world) {
    const int32_t* f = words(own) + ph * 8 + r;
    if (load_acquire_sys(f) < e) {
      const long long t0 = global_ns();
      while (load_acquire_sys(f) < e) {
        // give up after kWaitNs, or at once if a wait of this call (or an
        // earlier one: the bit stays set until the status word is cleared) did
        if (global_ns() - t0 > kWaitNs || (status && (load_volatile(status) & PS_DEV_WAIT_TIMEOUT))) {
          set_status(status, PS_DEV_WAIT_TIMEOUT);
          atomicAnd(&s_ok, 0);
          break;
        }
        __nanosleep(64);
      }
    }
  }
  __syncthreads();
  return s_ok != 0;
}

// CTA-wide: whether this CTA is the last of the grid to get here (the
// counter, word `word` of `own`'s header, is reset by that CTA).  Contains
// __syncthreads.
__device__ __forceinline__ bool last_cta(char* own, int word = kDoneWord) {
  __shared__ int s_last;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const int old = atomicAdd(words(own) + word, 1);
    s_last = old == static_cast<int>(gridDim.x) - 1;
    if (s_last) words(own)[word] = 0;
  }
  __syncthreads();
  return s_last != 0;
}

// Thread 0: record call e as completed on this rank.
__device__ __forceinline__ void close_call(char* own, int32_t e) {
  if (threadIdx.x == 0) {
    __threadfence();
    *reinterpret_cast<volatile int32_t*>(words(own) + kEpochWord) = e;
  }
}

}  // namespace peer
}  // namespace ps
