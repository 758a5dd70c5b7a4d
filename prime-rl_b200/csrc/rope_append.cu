// Fused rotary embedding + KV append for sm_100a.
//
// Replaces vLLM's fused custom op fused_rope_and_unified_kv_cache_update
// (vllm/compilation/passes/fusion/rope_kvcache_fusion.py:40-73), i.e. the
// backend hook AttentionImpl.do_rope_and_kv_cache_update
// (vllm/v1/attention/backend.py:815-841): rotate query and key in place, then
// write the rotated key and the value into the paged cache at slot_mapping.
//
// Arithmetic: the torch-native rotary embedding
// (vllm/model_executor/layers/rotary_embedding/base.py:140-181,
// common.py:144-180): cos/sin are cast to the model dtype, and
//   o1 = x1 * cos - x2 * sin,  o2 = x2 * cos + x1 * sin
// with every product and every sum rounded to the model dtype, as bf16/fp16
// tensor arithmetic does.  Products of two 16-bit floats are exact in fp32,
// so "fp32 multiply, round" equals the 16-bit multiply; the sum of the two
// rounded products is rounded once, as the 16-bit add is.  Results are
// bit-identical to the reference.
//
// Work: with 16-byte aligned rows and rotary_dim a multiple of 16, one thread
// per 8-element unit of a row (16-byte accesses, grid-stride); otherwise one
// warp per (token, head) row with element accesses.  A query row is rotated in
// place; a key row is rotated in place and written with the value row into
// the cache (slot < 0: no cache write).  HBM-bound: per token Hq*D*2*2 + Hkv*D*2*(2+1) + Hkv*D*2*2
// bytes (q read/write; k read/write/cache; v read/cache).
#include "ps_common.cuh"
#include "ps_launch.h"

namespace ps {

template <bool kBF16>
struct Half16;
template <>
struct Half16<true> {
  using T = __nv_bfloat16;
  using T2 = __nv_bfloat162;
  static __device__ __forceinline__ float f(T x) { return __bfloat162float(x); }
  static __device__ __forceinline__ T r(float x) { return __float2bfloat16_rn(x); }
};
template <>
struct Half16<false> {
  using T = __half;
  using T2 = __half2;
  static __device__ __forceinline__ float f(T x) { return __half2float(x); }
  static __device__ __forceinline__ T r(float x) { return __float2half_rn(x); }
};

// cos/sin entry as the model dtype: the cache holds fp32 or the model dtype
template <bool kBF16>
__device__ __forceinline__ float cs_value(const RopeArgs& a, int64_t row, int i) {
  using H = Half16<kBF16>;
  const char* base = a.cos_sin + row * a.cs_stride_bytes;
  if (a.cs_fp32) return H::f(H::r(reinterpret_cast<const float*>(base)[i]));
  return H::f(reinterpret_cast<const typename H::T*>(base)[i]);
}

// one rotated pair, rounding as the reference does
template <bool kBF16>
__device__ __forceinline__ void rotate_pair(float x1, float x2, float c, float s, float& o1,
                                            float& o2) {
  using H = Half16<kBF16>;
  const float a = H::f(H::r(__fmul_rn(x1, c))), b = H::f(H::r(__fmul_rn(x2, s)));
  const float d = H::f(H::r(__fmul_rn(x2, c))), e = H::f(H::r(__fmul_rn(x1, s)));
  o1 = H::f(H::r(__fsub_rn(a, b)));
  o2 = H::f(H::r(__fadd_rn(d, e)));
}

template <bool kBF16>
__global__ void __launch_bounds__(256) rope_kv_append_kernel(const RopeArgs a) {
  using H = Half16<kBF16>;
  using T = typename H::T;
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  const int heads = a.num_q_heads + a.num_kv_heads;
  const int64_t items = a.num_tokens * heads;
  const int half = a.rotary_dim / 2;
  const int D = a.head_size;
  asm volatile("griddepcontrol.wait;" ::: "memory");
  for (int64_t it = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5);
       it < items; it += warps) {
    const int64_t t = it / heads;
    const int hh = static_cast<int>(it - t * heads);
    const int64_t pos = __ldg(a.positions + t);
    if (pos < 0 || pos >= a.max_position) {
      if (lane == 0) set_status(a.status, PS_DEV_BAD_METADATA);
      continue;
    }
    const bool is_q = hh < a.num_q_heads;
    const int h = is_q ? hh : hh - a.num_q_heads;
    T* row = reinterpret_cast<T*>(is_q ? a.q + t * a.q_st + h * a.q_sh : a.k + t * a.k_st + h * a.k_sh);
    // destination row in the cache for a kv head (nullptr: none)
    T* krow = nullptr;
    T* vrow = nullptr;
    const T* vsrc = nullptr;
    if (!is_q) {
      const int64_t slot = __ldg(a.slot_mapping + t);
      if (slot >= a.num_slots) {
        if (lane == 0) set_status(a.status, PS_DEV_SLOT_OUT_OF_RANGE);
      } else if (slot >= 0) {
        const int64_t blk = slot / a.block_size, off = slot - blk * a.block_size;
        const int64_t o = blk * a.c_sblock + off * a.c_sslot + h * a.c_shead;
        krow = reinterpret_cast<T*>(a.key_cache + o);
        vrow = reinterpret_cast<T*>(a.value_cache + o);
        vsrc = reinterpret_cast<const T*>(a.v + t * a.v_st + h * a.v_sh);
      }
    }
    // rotated pairs: neox (i, i + half), GPT-J (2i, 2i + 1)
    for (int i = lane; i < half; i += 32) {
      const int i1 = a.neox ? i : 2 * i;
      const int i2 = a.neox ? i + half : 2 * i + 1;
      const float x1 = H::f(row[i1]), x2 = H::f(row[i2]);
      const float c = cs_value<kBF16>(a, pos, i), s = cs_value<kBF16>(a, pos, half + i);
      float o1, o2;
      rotate_pair<kBF16>(x1, x2, c, s, o1, o2);
      const T r1 = H::r(o1), r2 = H::r(o2);
      row[i1] = r1;
      row[i2] = r2;
      if (krow) {
        krow[i1] = r1;
        krow[i2] = r2;
      }
    }
    if (krow) {
      for (int i = a.rotary_dim + lane; i < D; i += 32) krow[i] = row[i];  // pass-through dims
      for (int i = lane; i < D; i += 32) vrow[i] = vsrc[i];
    }
  }
}

// Vector path: one thread per 8-element unit of a row, 16-byte accesses.
// Units: a query row has the rotation units only (pass-through dims stay in
// place); a kv row has its rotation units, the pass-through units (copied to
// the cache) and the value units (copied to the cache).  Neox: unit u rotates
// elements [8u, 8u+8) with [half+8u, half+8u+8); GPT-J: unit u holds the 4
// pairs of elements [8u, 8u+8).
template <bool kBF16>
__device__ __forceinline__ void unpack8(const uint4& v, float (&x)[8]) {
  using H = Half16<kBF16>;
  const typename H::T* e = reinterpret_cast<const typename H::T*>(&v);
#pragma unroll
  for (int i = 0; i < 8; ++i) x[i] = H::f(e[i]);
}
template <bool kBF16>
__device__ __forceinline__ uint4 pack8(const float (&x)[8]) {
  using H = Half16<kBF16>;
  uint4 v;
  typename H::T* e = reinterpret_cast<typename H::T*>(&v);
#pragma unroll
  for (int i = 0; i < 8; ++i) e[i] = H::r(x[i]);
  return v;
}
// n cos/sin entries from element offset i of a cache row, as model-dtype values
template <bool kBF16, bool kCsF32, int N>
__device__ __forceinline__ void load_cs(const char* row, int i, float (&c)[N]) {
  using H = Half16<kBF16>;
  if constexpr (kCsF32) {
    const float4* p = reinterpret_cast<const float4*>(row + static_cast<int64_t>(i) * 4);
#pragma unroll
    for (int j = 0; j < N / 4; ++j) {
      const float4 v = __ldg(p + j);
      c[4 * j] = H::f(H::r(v.x));
      c[4 * j + 1] = H::f(H::r(v.y));
      c[4 * j + 2] = H::f(H::r(v.z));
      c[4 * j + 3] = H::f(H::r(v.w));
    }
  } else if constexpr (N == 8) {
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(row + static_cast<int64_t>(i) * 2));
    unpack8<kBF16>(v, c);
  } else {
    const uint2 v = __ldg(reinterpret_cast<const uint2*>(row + static_cast<int64_t>(i) * 2));
    const typename H::T* e = reinterpret_cast<const typename H::T*>(&v);
#pragma unroll
    for (int j = 0; j < 4; ++j) c[j] = H::f(e[j]);
  }
}

template <bool kBF16, bool kNeox, bool kCsF32>
__global__ void __launch_bounds__(256) rope_kv_append_vec_kernel(const RopeArgs a) {
  const int D = a.head_size, rot = a.rotary_dim, half = rot / 2;
  const int ru = kNeox ? half / 8 : rot / 8;  // rotation units per row
  const int pu = (D - rot) / 8;                // pass-through units
  const int kvu = ru + pu + D / 8;             // + value units
  const int64_t q_units = a.num_tokens * a.num_q_heads * ru;
  const int64_t total = q_units + a.num_tokens * a.num_kv_heads * kvu;
  asm volatile("griddepcontrol.wait;" ::: "memory");
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    int64_t t;
    int h, u;
    bool is_q = i < q_units;
    if (is_q) {
      t = i / (static_cast<int64_t>(a.num_q_heads) * ru);
      const int r = static_cast<int>(i - t * a.num_q_heads * ru);
      h = r / ru;
      u = r - h * ru;
    } else {
      const int64_t j = i - q_units;
      t = j / (static_cast<int64_t>(a.num_kv_heads) * kvu);
      const int r = static_cast<int>(j - t * a.num_kv_heads * kvu);
      h = r / kvu;
      u = r - h * kvu;
    }
    const int64_t pos = __ldg(a.positions + t);
    if (pos < 0 || pos >= a.max_position) {
      set_status(a.status, PS_DEV_BAD_METADATA);
      continue;
    }
    char* row = is_q ? a.q + t * a.q_st + h * a.q_sh : a.k + t * a.k_st + h * a.k_sh;
    char* crow = nullptr;  // this kv row's key-cache row (value row at the same offset)
    if (!is_q) {
      const int64_t slot = __ldg(a.slot_mapping + t);
      if (slot >= a.num_slots) {
        set_status(a.status, PS_DEV_SLOT_OUT_OF_RANGE);
      } else if (slot >= 0) {
        const int64_t blk = slot / a.block_size, off = slot - blk * a.block_size;
        crow = a.key_cache + blk * a.c_sblock + off * a.c_sslot + h * a.c_shead;
      }
      if (u >= ru) {  // pass-through or value unit: a copy into the cache only
        if (crow == nullptr) continue;
        if (u < ru + pu) {
          const int e = rot + 8 * (u - ru);
          *reinterpret_cast<uint4*>(crow + e * 2) = *reinterpret_cast<const uint4*>(row + e * 2);
        } else {
          const int e = 8 * (u - ru - pu);
          const char* vrow = a.v + t * a.v_st + h * a.v_sh;
          *reinterpret_cast<uint4*>(crow + (a.value_cache - a.key_cache) + e * 2) =
              __ldg(reinterpret_cast<const uint4*>(vrow + e * 2));
        }
        continue;
      }
    }
    const char* csrow = a.cos_sin + pos * a.cs_stride_bytes;
    if constexpr (kNeox) {
      const int e1 = 8 * u, e2 = half + 8 * u;
      float x1[8], x2[8], c[8], s[8], o1[8], o2[8];
      unpack8<kBF16>(*reinterpret_cast<const uint4*>(row + e1 * 2), x1);
      unpack8<kBF16>(*reinterpret_cast<const uint4*>(row + e2 * 2), x2);
      load_cs<kBF16, kCsF32, 8>(csrow, 8 * u, c);
      load_cs<kBF16, kCsF32, 8>(csrow, half + 8 * u, s);
#pragma unroll
      for (int j = 0; j < 8; ++j) rotate_pair<kBF16>(x1[j], x2[j], c[j], s[j], o1[j], o2[j]);
      const uint4 v1 = pack8<kBF16>(o1), v2 = pack8<kBF16>(o2);
      *reinterpret_cast<uint4*>(row + e1 * 2) = v1;
      *reinterpret_cast<uint4*>(row + e2 * 2) = v2;
      if (crow) {
        *reinterpret_cast<uint4*>(crow + e1 * 2) = v1;
        *reinterpret_cast<uint4*>(crow + e2 * 2) = v2;
      }
    } else {
      const int e = 8 * u;
      float x[8], c[4], s[4], o[8];
      unpack8<kBF16>(*reinterpret_cast<const uint4*>(row + e * 2), x);
      load_cs<kBF16, kCsF32, 4>(csrow, 4 * u, c);
      load_cs<kBF16, kCsF32, 4>(csrow, half + 4 * u, s);
#pragma unroll
      for (int j = 0; j < 4; ++j) rotate_pair<kBF16>(x[2 * j], x[2 * j + 1], c[j], s[j], o[2 * j], o[2 * j + 1]);
      const uint4 v = pack8<kBF16>(o);
      *reinterpret_cast<uint4*>(row + e * 2) = v;
      if (crow) *reinterpret_cast<uint4*>(crow + e * 2) = v;
    }
  }
}

}  // namespace ps

int ps_launch_rope_kv_append(const ps::RopeArgs& a, int sm_count, int vec, cudaStream_t stream) {
  if (vec) {
    const int ru = a.neox ? a.rotary_dim / 16 : a.rotary_dim / 8;
    const int64_t units = a.num_tokens * (static_cast<int64_t>(a.num_q_heads) * ru +
                                          static_cast<int64_t>(a.num_kv_heads) *
                                              (ru + (a.head_size - a.rotary_dim) / 8 + a.head_size / 8));
    const int64_t blocks = (units + 255) / 256;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(blocks < 16LL * sm_count ? (blocks > 0 ? blocks : 1) : 16LL * sm_count));
    cfg.blockDim = dim3(256);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e;
#define PS_ROPE_VEC(BF, NX, CF) cudaLaunchKernelEx(&cfg, ps::rope_kv_append_vec_kernel<BF, NX, CF>, a)
    if (a.bf16)
      e = a.neox ? (a.cs_fp32 ? PS_ROPE_VEC(true, true, true) : PS_ROPE_VEC(true, true, false))
                 : (a.cs_fp32 ? PS_ROPE_VEC(true, false, true) : PS_ROPE_VEC(true, false, false));
    else
      e = a.neox ? (a.cs_fp32 ? PS_ROPE_VEC(false, true, true) : PS_ROPE_VEC(false, true, false))
                 : (a.cs_fp32 ? PS_ROPE_VEC(false, false, true) : PS_ROPE_VEC(false, false, false));
#undef PS_ROPE_VEC
    return static_cast<int>(e != cudaSuccess ? e : cudaGetLastError());
  }
  const int64_t items = a.num_tokens * (a.num_q_heads + a.num_kv_heads);
  const int64_t blocks = (items + 7) / 8;
  const int grid = static_cast<int>(blocks < 8LL * sm_count ? (blocks > 0 ? blocks : 1) : 8LL * sm_count);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(256);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = a.bf16 ? cudaLaunchKernelEx(&cfg, ps::rope_kv_append_kernel<true>, a)
                               : cudaLaunchKernelEx(&cfg, ps::rope_kv_append_kernel<false>, a);
  return static_cast<int>(e != cudaSuccess ? e : cudaGetLastError());
}
