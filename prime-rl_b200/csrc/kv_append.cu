// KV append: scatter the new tokens' key/value rows into the paged cache.
//
// Semantics of vLLM's reshape_and_cache_flash (NHD layout), as spelled out by
// its Triton twin vllm/v1/attention/ops/triton_reshape_and_cache_flash.py:
//   slot < 0 -> padding token, skipped                      (:46-48)
//   block = slot / block_size, offset = slot % block_size   (:50-51)
//   cache[block, offset, h, :] = src[t, h, :] for all heads (:78-87, :112-123)
//
// B200 layout: a CTA handles kAppendTokens tokens per iteration (grid-stride
// over tokens); its threads walk each token's 2 * num_heads head rows in
// VEC-byte vectors, head_size bytes contiguous per head row, so each warp
// moves whole 512-byte runs (16-byte vectors) on both the load and the store
// side.  The
// payload is never touched by arithmetic: the copy is bit-exact.
#include <climits>

#include "ps_common.cuh"
#include "ps_launch.h"

namespace ps {

template <int VEC>
struct VecT;
template <>
struct VecT<16> {
  using T = uint4;
};
template <>
struct VecT<8> {
  using T = uint2;
};
template <>
struct VecT<4> {
  using T = uint32_t;
};
template <>
struct VecT<2> {
  using T = uint16_t;
};

// Tokens per CTA iteration: their slot loads and row loads are all issued
// before any store, so a thread keeps kAppendTokens 16-byte rows in flight
// instead of one dependent slot -> row round trip per token.
constexpr int kAppendTokens = 4;

template <int VEC>
__global__ void __launch_bounds__(256) kv_append_kernel(AppendArgs a) {
  using V = typename VecT<VEC>::T;
  // let a programmatic dependent (the attention kernel) get scheduled now; it
  // still waits for this grid's completion before reading the cache
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  constexpr int U = kAppendTokens;
  const int per_tensor = a.num_heads * a.vecs_per_head;
  const int per_token = 2 * per_tensor;
  // a slot that passes the range check fits in 32 bits whenever the pool
  // does; the block / offset split is then a 32-bit division
  const bool narrow = a.num_slots <= INT32_MAX;
  for (int64_t t0 = static_cast<int64_t>(blockIdx.x) * U; t0 < a.num_tokens;
       t0 += static_cast<int64_t>(gridDim.x) * U) {
    int64_t slot[U];
#pragma unroll
    for (int u = 0; u < U; ++u) slot[u] = t0 + u < a.num_tokens ? __ldg(a.slot_mapping + t0 + u) : -1;
    for (int j = threadIdx.x; j < per_token; j += blockDim.x) {
      const bool is_v = j >= per_tensor;
      const int r = is_v ? j - per_tensor : j;
      const int h = r / a.vecs_per_head;
      const int c = r - h * a.vecs_per_head;
      const char* src0 = is_v ? a.value + h * a.val_sh : a.key + h * a.key_sh;
      const int64_t sst = is_v ? a.val_st : a.key_st;
      // every row of a token below num_tokens is readable (padding tokens
      // included), so the row loads do not wait for the slots
      V v[U];
#pragma unroll
      for (int u = 0; u < U; ++u)
        if (t0 + u < a.num_tokens) v[u] = __ldg(reinterpret_cast<const V*>(src0 + (t0 + u) * sst) + c);
      char* base = (is_v ? a.value_cache : a.key_cache) + h * a.c_shead;
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t sl = slot[u];
        if (sl < 0 || sl >= a.num_slots) continue;  // padding token / recorded below
        int64_t blk, off;
        if (narrow) {
          const uint32_t s32 = static_cast<uint32_t>(sl), bs = static_cast<uint32_t>(a.block_size);
          const uint32_t b32 = s32 / bs;
          blk = b32;
          off = s32 - b32 * bs;
        } else {
          blk = sl / a.block_size;
          off = sl - blk * a.block_size;
        }
        reinterpret_cast<V*>(base + blk * a.c_sblock + off * a.c_sslot)[c] = v[u];
      }
    }
    if (threadIdx.x == 0) {
#pragma unroll
      for (int u = 0; u < U; ++u)
        if (slot[u] >= a.num_slots) set_status(a.status, PS_DEV_SLOT_OUT_OF_RANGE);
    }
  }
}

}  // namespace ps

int ps_launch_kv_append(const ps::AppendArgs& a, int vec, int sm_count, cudaStream_t stream) {
  if (a.num_tokens == 0) return 0;
  const int threads = 256;
  int64_t blocks = (a.num_tokens + ps::kAppendTokens - 1) / ps::kAppendTokens;
  const int64_t cap = static_cast<int64_t>(sm_count) * 8;
  if (blocks > cap) blocks = cap;
  switch (vec) {
    case 16:
      ps::kv_append_kernel<16><<<static_cast<int>(blocks), threads, 0, stream>>>(a);
      break;
    case 8:
      ps::kv_append_kernel<8><<<static_cast<int>(blocks), threads, 0, stream>>>(a);
      break;
    case 4:
      ps::kv_append_kernel<4><<<static_cast<int>(blocks), threads, 0, stream>>>(a);
      break;
    default:
      ps::kv_append_kernel<2><<<static_cast<int>(blocks), threads, 0, stream>>>(a);
      break;
  }
  return static_cast<int>(cudaGetLastError());
}

namespace ps {

// fp8 (e4m3) cache: each 8-element piece of a head row (16 source bytes) is
// stored as 8 e4m3 codes of x / scale -- the fp8 branch of the Triton twin
// (:93-110: key / k_scale, value / v_scale, converted to the cache's fp8 type
// by the store), rounded to the nearest e4m3 (ties to even) and saturating
// at +-448.  vecs_per_head counts 8-element pieces.
template <bool kBF16>
__global__ void __launch_bounds__(256) kv_append_fp8_kernel(AppendArgs a, const float* k_scale,
                                                            const float* v_scale) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const float ks = k_scale ? __ldg(k_scale) : 1.f;
  const float vs = v_scale ? __ldg(v_scale) : 1.f;
  const int per_tensor = a.num_heads * a.vecs_per_head;
  const int per_token = 2 * per_tensor;
  for (int64_t t = blockIdx.x; t < a.num_tokens; t += gridDim.x) {
    const int64_t slot = __ldg(a.slot_mapping + t);
    if (slot < 0) continue;  // padding token
    if (slot >= a.num_slots) {
      if (threadIdx.x == 0) set_status(a.status, PS_DEV_SLOT_OUT_OF_RANGE);
      continue;
    }
    const int64_t blk = slot / a.block_size;
    const int64_t off = slot - blk * a.block_size;
    const int64_t dst_tok = blk * a.c_sblock + off * a.c_sslot;
    for (int j = threadIdx.x; j < per_token; j += blockDim.x) {
      const bool is_v = j >= per_tensor;
      const int r = is_v ? j - per_tensor : j;
      const int h = r / a.vecs_per_head;
      const int c = r - h * a.vecs_per_head;
      const char* src = is_v ? a.value + t * a.val_st + h * a.val_sh
                             : a.key + t * a.key_st + h * a.key_sh;
      char* dst = (is_v ? a.value_cache : a.key_cache) + dst_tok + h * a.c_shead;
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(src) + c);
      reinterpret_cast<uint2*>(dst)[c] = quantize8_e4m3<kBF16>(v, is_v ? vs : ks);
    }
  }
}

}  // namespace ps

int ps_launch_kv_append_fp8(const ps::AppendArgs& a, const float* k_scale, const float* v_scale,
                            int dtype_bf16, int sm_count, cudaStream_t stream) {
  if (a.num_tokens == 0) return 0;
  int64_t blocks = (a.num_tokens + ps::kAppendTokens - 1) / ps::kAppendTokens;
  const int64_t cap = static_cast<int64_t>(sm_count) * 8;
  if (blocks > cap) blocks = cap;
  if (dtype_bf16)
    ps::kv_append_fp8_kernel<true><<<static_cast<int>(blocks), 256, 0, stream>>>(a, k_scale, v_scale);
  else
    ps::kv_append_fp8_kernel<false><<<static_cast<int>(blocks), 256, 0, stream>>>(a, k_scale, v_scale);
  return static_cast<int>(cudaGetLastError());
}

namespace ps {

// The pages of an fp8 cache that a batch of sequences reads, dequantized into
// a 16-bit scratch cache for kernels that take 16-bit pages (chunked
// prefill): page p < ceil(seq_lens[b] / block_size) of sequence b (cache
// block block_table[b][p]) becomes scratch block b * max_pages + p, each
// element code * scale (fp32) rounded to the model dtype.  Cache blocks are
// contiguous [block_size, num_kv_heads, 128] bytes; 16 codes per thread step.
template <bool kBF16>
__global__ void __launch_bounds__(256) kv_dequant_gather_kernel(const DequantArgs a) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const float ks = a.k_scale ? __ldg(a.k_scale) : 1.f;
  const float vs = a.v_scale ? __ldg(a.v_scale) : 1.f;
  const int64_t cpb = a.block_bytes / 16;  // 16-code chunks per block
  const int64_t units = static_cast<int64_t>(a.num_seqs) * a.max_pages * 2 * cpb;
  const int64_t gstride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t u = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; u < units; u += gstride) {
    const int64_t c = u % cpb;
    const int64_t rest = u / cpb;
    const int which = static_cast<int>(rest & 1);  // 0 key, 1 value
    const int64_t page = rest >> 1;                // b * max_pages + p
    const int b = static_cast<int>(page / a.max_pages);
    const int p = static_cast<int>(page - static_cast<int64_t>(b) * a.max_pages);
    const int L = __ldg(a.seq_lens + b);
    if (p * a.block_size >= L) continue;
    if (p >= a.max_blocks_per_seq) {
      if (c == 0 && which == 0) set_status(a.status, PS_DEV_BAD_METADATA);
      continue;
    }
    const int blk = __ldg(a.block_table + static_cast<int64_t>(b) * a.bt_stride + p);
    if (blk < 0 || blk >= a.num_blocks) {
      if (c == 0 && which == 0) set_status(a.status, PS_DEV_BLOCK_OUT_OF_RANGE);
      continue;
    }
    const uint4 codes = __ldg(reinterpret_cast<const uint4*>(
        (which ? a.value_cache : a.key_cache) + blk * a.c_sblock + c * 16));
    const float s = which ? vs : ks;
    const uint32_t w[4] = {codes.x, codes.y, codes.z, codes.w};
    uint32_t o[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t lo16 = e4m3x2_to_f16x2(w[i]);
      const uint32_t hi16 = e4m3x2_to_f16x2(w[i] >> 16);
      const float2 lo = __half22float2(*reinterpret_cast<const __half2*>(&lo16));
      const float2 hi = __half22float2(*reinterpret_cast<const __half2*>(&hi16));
      o[2 * i] = pack2<kBF16>(lo.x * s, lo.y * s);
      o[2 * i + 1] = pack2<kBF16>(hi.x * s, hi.y * s);
    }
    uint4* dst = reinterpret_cast<uint4*>((which ? a.out_value : a.out_key) + (page * a.block_bytes + c * 16) * 2);
    dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
    dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
  }
}

}  // namespace ps

int ps_launch_kv_dequant_gather(const ps::DequantArgs& a, int dtype_bf16, int sm_count,
                                cudaStream_t stream) {
  const int64_t units = static_cast<int64_t>(a.num_seqs) * a.max_pages * 2 * (a.block_bytes / 16);
  if (units == 0) return 0;
  int64_t g = (units + 255) / 256;
  const int64_t cap = 8LL * sm_count;
  if (g > cap) g = cap;
  if (dtype_bf16)
    ps::kv_dequant_gather_kernel<true><<<static_cast<unsigned>(g), 256, 0, stream>>>(a);
  else
    ps::kv_dequant_gather_kernel<false><<<static_cast<unsigned>(g), 256, 0, stream>>>(a);
  return static_cast<int>(cudaGetLastError());
}
