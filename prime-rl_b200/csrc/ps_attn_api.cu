// C ABI of libps_attn.so: argument validation, TMA descriptor encoding and
// kernel launches.  Declarations and contracts live in include/ps_attn.h.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "ps_common.cuh"
#include "ps_launch.h"

namespace {

thread_local char g_err[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(PS_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

// SM count of the current device, cached per device ordinal.
int sm_count_current(int* out_dev) {
  static std::mutex mu;
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  if (out_dev) *out_dev = dev;
  std::lock_guard<std::mutex> lk(mu);
  if (dev < 64 && cache[dev] > 0) return cache[dev];
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return -1;
  if (dev < 64) cache[dev] = n;
  return n;
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// Tensor map over one cache half viewed as [num_blocks][block_size][Hkv][128]
// 16-bit elements; box = one 16-token page of one head, 64 dims (128 B) wide,
// 128-byte swizzle.  elem_bytes = 1 (fp8 cache): the box is all 128 dims,
// again 128 bytes wide.  L2 promotion: 256 B for a 16-bit cache (a head's row,
// whose other half the next box reads), 128 B for fp8, whose head row is 128 B:
// a 256-byte promotion would pull in the neighbouring head's row, which
// another warp streams much later (measured: 1.31x the algorithmic DRAM bytes
// and a 23% slower config-5 step).
int make_page_map(CUtensorMap* map, const void* base, int64_t num_blocks, int block_size,
                  int num_kv_heads, int64_t s_block, int64_t s_slot, int64_t s_head,
                  int elem_bytes = 2) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(PS_ERR_CUDA, "cuTensorMapEncodeTiled unavailable from the driver");
  const cuuint64_t eb = static_cast<cuuint64_t>(elem_bytes);
  cuuint64_t dims[4] = {128, static_cast<cuuint64_t>(num_kv_heads),
                        static_cast<cuuint64_t>(block_size), static_cast<cuuint64_t>(num_blocks)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(s_head) * eb, static_cast<cuuint64_t>(s_slot) * eb,
                           static_cast<cuuint64_t>(s_block) * eb};
  cuuint32_t box[4] = {elem_bytes == 1 ? 128u : 64u, 1, 16, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(map, elem_bytes == 1 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_UINT16,
                  4, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  elem_bytes == 1 ? CU_TENSOR_MAP_L2_PROMOTION_L2_128B : CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(PS_ERR_INVALID_ARGUMENT,
                "cuTensorMapEncodeTiled failed (%d): cache strides must be multiples of 16 "
                "bytes and the base 16-byte aligned",
                static_cast<int>(r));
  return PS_OK;
}

// Tensor map over q viewed as [num_tokens][num_q_heads][128] 16-bit elements;
// box = 64 dims x `group` heads x `tokens` tokens, 128-byte swizzle.  Its smem
// image is row (token * group + head) of 128 bytes: the K-major SW128 layout.
int make_q_map(CUtensorMap* map, const void* q, int64_t num_tokens, int num_q_heads,
               int64_t s_token, int64_t s_head, int group, int tokens) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(PS_ERR_CUDA, "cuTensorMapEncodeTiled unavailable from the driver");
  cuuint64_t dims[3] = {128, static_cast<cuuint64_t>(num_q_heads), static_cast<cuuint64_t>(num_tokens)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(s_head) * 2, static_cast<cuuint64_t>(s_token) * 2};
  cuuint32_t box[3] = {64, static_cast<cuuint32_t>(group), static_cast<cuuint32_t>(tokens)};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, const_cast<void*>(q), dims, strides, box,
                  estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(PS_ERR_INVALID_ARGUMENT, "q tensor map rejected (%d): strides must be multiples of 16 bytes",
                static_cast<int>(r));
  return PS_OK;
}

bool aligned(const void* p, int bytes) {
  return (reinterpret_cast<uintptr_t>(p) % static_cast<uintptr_t>(bytes)) == 0;
}

int64_t round_up(int64_t x, int64_t m) { return (x + m - 1) / m * m; }

// Decode workspace layout.  Every offset is independent of the call's
// num_seqs, and the plain and cascade layouts agree on everything but the
// record size, so one buffer (sized for the larger use) serves calls of either
// kind with any batch size up to the one it was sized for:
//   [0, 256)                 status word; bytes 16..23: prefill unit scheduler
//   [256, 256 + C)           counters, kDecodeMaxSeqs * num_kv_heads int32
//   [.., + C)                prefix-segment counters (cascade)
//   [..., ...)               partial records, one per split slot:
//                            kg * 128 fp32 output rows, then kg fp32 LSEs
//                            (kg = 8 or 16 by GQA group; 16 in cascade mode)
// The counters must be zero before the first call; every call leaves them zero.
struct DecodeWorkspaceLayout {
  int64_t counters_off, pre_counters_off, part_off, record_bytes, total;
};

DecodeWorkspaceLayout decode_layout(int num_seqs, int num_q_heads, int num_kv_heads, int sm_count,
                                    bool cascade, bool fp8 = false) {
  const int group = num_q_heads / num_kv_heads;
  const int kg = (group <= 8 && !cascade) ? 8 : 16;
  const int64_t slots =
      ps_decode_partial_slots(num_seqs, num_kv_heads, sm_count, cascade ? 1 : 0, fp8 ? 1 : 0);
  const int64_t counter_bytes = static_cast<int64_t>(ps::kDecodeMaxSeqs) * num_kv_heads * 4;
  DecodeWorkspaceLayout l;
  l.counters_off = 256;
  l.pre_counters_off = round_up(l.counters_off + counter_bytes, 256);
  l.part_off = round_up(l.pre_counters_off + counter_bytes, 256);
  l.record_bytes = static_cast<int64_t>(kg) * 129 * 4;
  l.total = round_up(l.part_off + slots * l.record_bytes, 256);
  return l;
}

int validate_problem(const ps_paged_problem* pr, bool decode) {
  if (!pr) return fail(PS_ERR_INVALID_ARGUMENT, "problem is NULL");
  if (pr->num_seqs < 0) return fail(PS_ERR_INVALID_ARGUMENT, "num_seqs < 0");
  if (pr->num_seqs == 0) return PS_OK;
  if (!pr->q || !pr->key_cache || !pr->value_cache || !pr->block_table || !pr->seq_lens ||
      !pr->out)
    return fail(PS_ERR_INVALID_ARGUMENT, "a required pointer is NULL");
  if (!decode && !pr->query_start_loc)
    return fail(PS_ERR_INVALID_ARGUMENT, "chunked prefill needs query_start_loc");
  if (pr->dtype != PS_DTYPE_BF16 && pr->dtype != PS_DTYPE_FP16)
    return fail(PS_ERR_UNSUPPORTED, "attention supports fp16 and bf16 only (dtype %d)", pr->dtype);
  if (pr->head_size != 128)
    return fail(PS_ERR_UNSUPPORTED, "head_size %d unsupported (this build: 128)", pr->head_size);
  if (pr->block_size <= 0 || pr->block_size % 16 != 0 || pr->block_size > 256)
    return fail(PS_ERR_INVALID_ARGUMENT, "block_size %d must be a multiple of 16 in [16, 256]",
                pr->block_size);
  if (pr->num_kv_heads <= 0 || pr->num_q_heads <= 0 || pr->num_q_heads % pr->num_kv_heads != 0)
    return fail(PS_ERR_INVALID_ARGUMENT, "num_q_heads %d must be a positive multiple of num_kv_heads %d",
                pr->num_q_heads, pr->num_kv_heads);
  const int group = pr->num_q_heads / pr->num_kv_heads;
  if (group > 16)
    return fail(PS_ERR_UNSUPPORTED, "GQA group %d > 16 unsupported", group);
  if (pr->num_blocks <= 0 || pr->num_blocks > INT32_MAX)
    return fail(PS_ERR_INVALID_ARGUMENT, "num_blocks out of range");
  if (pr->max_blocks_per_seq < 0 || pr->block_table_stride < pr->max_blocks_per_seq)
    return fail(PS_ERR_INVALID_ARGUMENT, "block_table_stride < max_blocks_per_seq");
  if (pr->kv_cache_dtype != PS_KV_AUTO && pr->kv_cache_dtype != PS_KV_FP8_E4M3)
    return fail(PS_ERR_INVALID_ARGUMENT, "kv_cache_dtype %d unknown", pr->kv_cache_dtype);
  // 16-byte rows for TMA / vector access (strides in cache elements)
  const int64_t cv = pr->kv_cache_dtype == PS_KV_FP8_E4M3 ? 16 : 8;
  if (!aligned(pr->key_cache, 16) || !aligned(pr->value_cache, 16) ||
      pr->cache_stride_head % cv || pr->cache_stride_slot % cv || pr->cache_stride_block % cv)
    return fail(PS_ERR_INVALID_ARGUMENT, "cache base/strides must be 16-byte aligned");
  if (!aligned(pr->q, 16) || pr->q_stride_head % 8 || pr->q_stride_token % 8)
    return fail(PS_ERR_INVALID_ARGUMENT, "q base/strides must be 16-byte aligned");
  if (!aligned(pr->out, 16) || pr->out_stride_head % 8 || pr->out_stride_token % 8)
    return fail(PS_ERR_INVALID_ARGUMENT, "out base/strides must be 16-byte aligned");
  if (!(pr->softmax_scale > 0.f))
    return fail(PS_ERR_INVALID_ARGUMENT, "softmax_scale must be positive");
  return PS_OK;
}

int decode_impl(const ps_paged_problem* pr, const void* plan, int64_t plan_bytes, void* workspace,
                int64_t workspace_bytes, void* stream, bool cascade,
                const ps_head_gather_problem* gather = nullptr) {
  int rc = validate_problem(pr, true);
  if (rc != PS_OK) return rc;
  if (pr->num_seqs == 0) return PS_OK;
  if (pr->num_seqs > ps::kDecodeMaxSeqs)
    return fail(PS_ERR_UNSUPPORTED, "num_seqs %d > %d per decode launch", pr->num_seqs,
                ps::kDecodeMaxSeqs);
  int dev = 0;
  const int sms = sm_count_current(&dev);
  if (sms <= 0) return fail(PS_ERR_CUDA, "no CUDA device");
  if (cascade) {
    if (pr->num_seqs > ps::kCascadeMaxSeqs)
      return fail(PS_ERR_UNSUPPORTED, "num_seqs %d > %d per cascade decode launch", pr->num_seqs,
                  ps::kCascadeMaxSeqs);
    if (pr->num_q_heads / pr->num_kv_heads > 8)
      return fail(PS_ERR_UNSUPPORTED, "cascade decode needs a GQA group <= 8");
    if (!plan || !aligned(plan, 16) ||
        plan_bytes < ps_cascade_plan_words(pr->num_seqs) * static_cast<int64_t>(sizeof(int32_t)))
      return fail(PS_ERR_INVALID_ARGUMENT, "cascade plan must be >= %lld bytes, 16-byte aligned",
                  static_cast<long long>(ps_cascade_plan_words(pr->num_seqs) * 4));
  }
  const bool fp8 = pr->kv_cache_dtype == PS_KV_FP8_E4M3;
  if (fp8 && cascade) return fail(PS_ERR_UNSUPPORTED, "cascade decode over an fp8 cache is not built");
  const DecodeWorkspaceLayout lay =
      decode_layout(pr->num_seqs, pr->num_q_heads, pr->num_kv_heads, sms, cascade, fp8);
  if (!workspace || workspace_bytes < lay.total || !aligned(workspace, 256))
    return fail(PS_ERR_WORKSPACE, "decode workspace must be >= %lld bytes, 256-byte aligned",
                static_cast<long long>(lay.total));
  CUtensorMap kmap, vmap;
  rc = make_page_map(&kmap, pr->key_cache, pr->num_blocks, pr->block_size, pr->num_kv_heads,
                     pr->cache_stride_block, pr->cache_stride_slot, pr->cache_stride_head, fp8 ? 1 : 2);
  if (rc != PS_OK) return rc;
  rc = make_page_map(&vmap, pr->value_cache, pr->num_blocks, pr->block_size, pr->num_kv_heads,
                     pr->cache_stride_block, pr->cache_stride_slot, pr->cache_stride_head, fp8 ? 1 : 2);
  if (rc != PS_OK) return rc;
  char* ws = static_cast<char*>(workspace);
  ps::DecodeParams p = {};  // every optional feature off
  p.q = pr->q;
  p.q_st = pr->q_stride_token;
  p.q_sh = pr->q_stride_head;
  p.block_table = pr->block_table;
  p.bt_stride = pr->block_table_stride;
  p.max_blocks_per_seq = pr->max_blocks_per_seq;
  p.seq_lens = pr->seq_lens;
  p.qsl = pr->query_start_loc;
  p.num_seqs = pr->num_seqs;
  p.out = pr->out;
  p.o_st = pr->out_stride_token;
  p.o_sh = pr->out_stride_head;
  p.lse = pr->lse;
  p.lse_sh = pr->lse_stride_head;
  p.lse_st = pr->lse_stride_token;
  p.num_q_heads = pr->num_q_heads;
  p.num_kv_heads = pr->num_kv_heads;
  p.group = pr->num_q_heads / pr->num_kv_heads;
  p.block_size = pr->block_size;
  p.num_blocks = pr->num_blocks;
  p.scale_log2 = pr->softmax_scale * 1.4426950408889634f;
  p.status = reinterpret_cast<int32_t*>(ws);
  p.counters = reinterpret_cast<int32_t*>(ws + lay.counters_off);
  p.part = reinterpret_cast<float*>(ws + lay.part_off);
  p.num_part_slots =
      ps_decode_partial_slots(pr->num_seqs, pr->num_kv_heads, sms, cascade ? 1 : 0, fp8 ? 1 : 0);
  p.pre_counters = reinterpret_cast<int32_t*>(ws + lay.pre_counters_off);
  p.cas_num_groups = nullptr;
  p.cas_seq_group = p.cas_group_first = p.cas_group_size = p.cas_group_pages = nullptr;
  p.cas_max_groups = 0;
  if (cascade) {
    const int32_t* w = static_cast<const int32_t*>(plan);
    const int gm = pr->num_seqs / 2 > 1 ? pr->num_seqs / 2 : 1;
    p.cas_num_groups = w;
    p.cas_seq_group = w + 32;
    p.cas_group_first = p.cas_seq_group + pr->num_seqs;
    p.cas_group_size = p.cas_group_first + gm;
    p.cas_group_pages = p.cas_group_size + gm;
    p.cas_max_groups = gm;
  }
  p.new_key = pr->new_key;
  p.new_value = pr->new_value;
  p.nk_st = pr->new_key_stride_token;
  p.nk_sh = pr->new_key_stride_head;
  p.nv_st = pr->new_value_stride_token;
  p.nv_sh = pr->new_value_stride_head;
  p.slot_mapping = pr->slot_mapping;
  p.key_cache = const_cast<void*>(pr->key_cache);
  p.value_cache = const_cast<void*>(pr->value_cache);
  p.c_sblock = pr->cache_stride_block;
  p.c_sslot = pr->cache_stride_slot;
  p.c_shead = pr->cache_stride_head;
  p.k_scale = pr->k_scale;
  p.v_scale = pr->v_scale;
  if (pr->new_key != nullptr) {
    if (!pr->new_value || !pr->slot_mapping)
      return fail(PS_ERR_INVALID_ARGUMENT, "fused append needs new_key, new_value and slot_mapping");
    if (!aligned(pr->new_key, 16) || !aligned(pr->new_value, 16) || pr->new_key_stride_token % 8 ||
        pr->new_key_stride_head % 8 || pr->new_value_stride_token % 8 || pr->new_value_stride_head % 8)
      return fail(PS_ERR_INVALID_ARGUMENT, "new key/value rows must be 16-byte aligned");
  }
  if (gather != nullptr) {
    const int hq = gather->hq_local;
    p.gather_world = gather->world;
    p.gather_rank = gather->rank;
    p.gather_hq_local = hq;
    p.gather_tokens = gather->num_tokens;
    p.gather_row_st = static_cast<int64_t>(gather->world) * hq * 256;
    for (int r = 0; r < gather->world; ++r) {
      char* slab = static_cast<char*>(gather->slabs[r]);
      p.gather_slab[r] = slab;
      p.gather_rows[r] = r == gather->rank
                             ? nullptr
                             : slab + ps::kDecodeGatherRowsOffset + static_cast<int64_t>(gather->rank) * hq * 256;
    }
    p.gather_out = static_cast<char*>(gather->out);
    p.gather_o_st = gather->out_stride_token * 2;
    p.gather_o_sh = gather->out_stride_head * 2;
    p.gather_status = gather->status;
  }
  const int e = ps_launch_paged_decode(p, kmap, vmap, pr->dtype == PS_DTYPE_BF16, sms,
                                       static_cast<cudaStream_t>(stream), fp8 ? 1 : 0);
  if (e != 0) return cuda_fail(static_cast<cudaError_t>(e), "paged_decode launch");
  return PS_OK;
}

}  // namespace

int ps_set_last_error(int code, const char* msg) { return fail(code, "%s", msg); }

int64_t ps_decode_workspace_bytes(int num_seqs, int num_q_heads, int num_kv_heads, int sm_count,
                                  int cascade, int fp8) {
  return decode_layout(num_seqs, num_q_heads, num_kv_heads, sm_count, cascade != 0, fp8 != 0).total;
}

extern "C" {

int ps_abi_version(void) { return PS_ATTN_ABI_VERSION; }

const char* ps_last_error(void) { return g_err; }

int ps_kv_append(const void* key, int64_t key_stride_token, int64_t key_stride_head,
                 const void* value, int64_t value_stride_token, int64_t value_stride_head,
                 void* key_cache, void* value_cache, int64_t cache_stride_block,
                 int64_t cache_stride_slot, int64_t cache_stride_head, int64_t num_blocks,
                 const int64_t* slot_mapping, int64_t num_tokens, int num_kv_heads, int head_size,
                 int block_size, int elem_bytes, int32_t* status, void* stream) {
  if (num_tokens < 0) return fail(PS_ERR_INVALID_ARGUMENT, "num_tokens < 0");
  if (num_tokens == 0) return PS_OK;
  if (!key || !value || !key_cache || !value_cache || !slot_mapping)
    return fail(PS_ERR_INVALID_ARGUMENT, "a required pointer is NULL");
  if (elem_bytes != 2 && elem_bytes != 4 && elem_bytes != 1)
    return fail(PS_ERR_UNSUPPORTED, "elem_bytes %d unsupported", elem_bytes);
  if (num_kv_heads <= 0 || head_size <= 0 || block_size <= 0 || num_blocks <= 0)
    return fail(PS_ERR_INVALID_ARGUMENT, "non-positive shape");
  const int64_t row = static_cast<int64_t>(head_size) * elem_bytes;
  // widest vector every address and stride admits
  int vec = 16;
  auto ok = [&](int v) {
    if (row % v) return false;
    const void* ps[4] = {key, value, key_cache, value_cache};
    for (const void* p : ps)
      if (!aligned(p, v)) return false;
    const int64_t st[7] = {key_stride_token, key_stride_head, value_stride_token, value_stride_head,
                           cache_stride_block, cache_stride_slot, cache_stride_head};
    for (int64_t s : st)
      if ((s * elem_bytes) % v) return false;
    return true;
  };
  while (vec > 1 && !ok(vec)) vec >>= 1;
  if (vec < 2) return fail(PS_ERR_INVALID_ARGUMENT, "rows are not 2-byte aligned");
  int dev = 0;
  const int sms = sm_count_current(&dev);
  if (sms <= 0) return fail(PS_ERR_CUDA, "no CUDA device");
  ps::AppendArgs a;
  a.key = static_cast<const char*>(key);
  a.value = static_cast<const char*>(value);
  a.key_cache = static_cast<char*>(key_cache);
  a.value_cache = static_cast<char*>(value_cache);
  a.slot_mapping = slot_mapping;
  a.key_st = key_stride_token * elem_bytes;
  a.key_sh = key_stride_head * elem_bytes;
  a.val_st = value_stride_token * elem_bytes;
  a.val_sh = value_stride_head * elem_bytes;
  a.c_sblock = cache_stride_block * elem_bytes;
  a.c_sslot = cache_stride_slot * elem_bytes;
  a.c_shead = cache_stride_head * elem_bytes;
  a.num_slots = num_blocks * block_size;
  a.num_tokens = num_tokens;
  a.num_heads = num_kv_heads;
  a.block_size = block_size;
  a.vecs_per_head = static_cast<int32_t>(row / vec);
  a.status = status;
  const int e = ps_launch_kv_append(a, vec, sms, static_cast<cudaStream_t>(stream));
  if (e != 0) return cuda_fail(static_cast<cudaError_t>(e), "kv_append launch");
  return PS_OK;
}

int ps_kv_append_fp8(const void* key, int64_t key_stride_token, int64_t key_stride_head,
                     const void* value, int64_t value_stride_token, int64_t value_stride_head,
                     void* key_cache, void* value_cache, int64_t cache_stride_block,
                     int64_t cache_stride_slot, int64_t cache_stride_head, int64_t num_blocks,
                     const int64_t* slot_mapping, int64_t num_tokens, int32_t num_kv_heads,
                     int32_t head_size, int32_t block_size, int32_t dtype, const float* k_scale,
                     const float* v_scale, int32_t* status, void* stream) {
  if (num_tokens < 0) return fail(PS_ERR_INVALID_ARGUMENT, "num_tokens < 0");
  if (num_tokens == 0) return PS_OK;
  if (!key || !value || !key_cache || !value_cache || !slot_mapping)
    return fail(PS_ERR_INVALID_ARGUMENT, "a required pointer is NULL");
  if (dtype != PS_DTYPE_BF16 && dtype != PS_DTYPE_FP16)
    return fail(PS_ERR_UNSUPPORTED, "fp8 append takes fp16 or bf16 rows (dtype %d)", dtype);
  if (num_kv_heads <= 0 || head_size <= 0 || head_size % 8 || block_size <= 0 || num_blocks <= 0)
    return fail(PS_ERR_INVALID_ARGUMENT, "non-positive shape or head_size not a multiple of 8");
  if (!aligned(key, 16) || !aligned(value, 16) || key_stride_token % 8 || key_stride_head % 8 ||
      value_stride_token % 8 || value_stride_head % 8)
    return fail(PS_ERR_INVALID_ARGUMENT, "key/value rows must be 16-byte aligned");
  if (!aligned(key_cache, 8) || !aligned(value_cache, 8) || cache_stride_block % 8 ||
      cache_stride_slot % 8 || cache_stride_head % 8)
    return fail(PS_ERR_INVALID_ARGUMENT, "fp8 cache rows must be 8-byte aligned");
  int dev = 0;
  const int sms = sm_count_current(&dev);
  if (sms <= 0) return fail(PS_ERR_CUDA, "no CUDA device");
  ps::AppendArgs a;
  a.key = static_cast<const char*>(key);
  a.value = static_cast<const char*>(value);
  a.key_cache = static_cast<char*>(key_cache);
  a.value_cache = static_cast<char*>(value_cache);
  a.slot_mapping = slot_mapping;
  a.key_st = key_stride_token * 2;
  a.key_sh = key_stride_head * 2;
  a.val_st = value_stride_token * 2;
  a.val_sh = value_stride_head * 2;
  a.c_sblock = cache_stride_block;
  a.c_sslot = cache_stride_slot;
  a.c_shead = cache_stride_head;
  a.num_slots = num_blocks * block_size;
  a.num_tokens = num_tokens;
  a.num_heads = num_kv_heads;
  a.block_size = block_size;
  a.vecs_per_head = head_size / 8;
  a.status = status;
  const int e = ps_launch_kv_append_fp8(a, k_scale, v_scale, dtype == PS_DTYPE_BF16, sms,
                                        static_cast<cudaStream_t>(stream));
  if (e != 0) return cuda_fail(static_cast<cudaError_t>(e), "kv_append_fp8 launch");
  return PS_OK;
}

int64_t ps_paged_decode_workspace_size(int32_t num_seqs, int32_t num_q_heads,
                                       int32_t num_kv_heads, int32_t head_size) {
  if (num_seqs < 0 || num_kv_heads <= 0 || num_q_heads <= 0 || head_size != 128) {
    fail(PS_ERR_INVALID_ARGUMENT, "workspace size: bad shape");
    return -1;
  }
  const int sms = sm_count_current(nullptr);
  if (sms <= 0) {
    fail(PS_ERR_CUDA, "no CUDA device");
    return -1;
  }
  // large enough for the 16-bit-cache and the fp8-cache kernels
  const int64_t a = decode_layout(num_seqs, num_q_heads, num_kv_heads, sms, false, false).total;
  const int64_t b = decode_layout(num_seqs, num_q_heads, num_kv_heads, sms, false, true).total;
  return a > b ? a : b;
}

int ps_paged_decode(const ps_paged_problem* pr, void* workspace, int64_t workspace_bytes,
                    void* stream) {
  return decode_impl(pr, nullptr, 0, workspace, workspace_bytes, stream, false);
}

int64_t ps_cascade_plan_bytes(int32_t num_seqs) {
  if (num_seqs < 0 || num_seqs > ps::kCascadeMaxSeqs) {
    fail(PS_ERR_INVALID_ARGUMENT, "cascade plan: num_seqs %d outside [0, %d]", num_seqs,
         ps::kCascadeMaxSeqs);
    return -1;
  }
  return ps_cascade_plan_words(num_seqs) * static_cast<int64_t>(sizeof(int32_t));
}

int ps_cascade_plan_build(const ps_paged_problem* pr, int32_t min_shared_pages, void* plan,
                          int64_t plan_bytes, void* stream) {
  if (!pr || !plan) return fail(PS_ERR_INVALID_ARGUMENT, "problem or plan is NULL");
  if (pr->num_seqs < 0 || pr->num_seqs > ps::kCascadeMaxSeqs)
    return fail(PS_ERR_UNSUPPORTED, "cascade plan: num_seqs %d outside [0, %d]", pr->num_seqs,
                ps::kCascadeMaxSeqs);
  if (!aligned(plan, 16) ||
      plan_bytes < ps_cascade_plan_words(pr->num_seqs) * static_cast<int64_t>(sizeof(int32_t)))
    return fail(PS_ERR_INVALID_ARGUMENT, "cascade plan must be >= %lld bytes, 16-byte aligned",
                static_cast<long long>(ps_cascade_plan_words(pr->num_seqs) * 4));
  if (min_shared_pages < 1) return fail(PS_ERR_INVALID_ARGUMENT, "min_shared_pages must be >= 1");
  if (pr->num_seqs == 0) {
    const cudaError_t e = cudaMemsetAsync(plan, 0, 4, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? PS_OK : cuda_fail(e, "cascade plan");
  }
  if (!pr->block_table || !pr->seq_lens) return fail(PS_ERR_INVALID_ARGUMENT, "a required pointer is NULL");
  if (pr->block_size <= 0 || pr->block_size % 16 != 0 || pr->block_size > 256)
    return fail(PS_ERR_INVALID_ARGUMENT, "block_size %d must be a multiple of 16 in [16, 256]",
                pr->block_size);
  if (pr->num_kv_heads <= 0 || pr->num_q_heads <= 0 || pr->num_q_heads % pr->num_kv_heads != 0)
    return fail(PS_ERR_INVALID_ARGUMENT, "num_q_heads %d must be a positive multiple of num_kv_heads %d",
                pr->num_q_heads, pr->num_kv_heads);
  if (pr->max_blocks_per_seq < 0 || pr->block_table_stride < pr->max_blocks_per_seq)
    return fail(PS_ERR_INVALID_ARGUMENT, "block_table_stride < max_blocks_per_seq");
  ps::PlanArgs a;
  a.block_table = pr->block_table;
  a.bt_stride = pr->block_table_stride;
  a.max_blocks_per_seq = pr->max_blocks_per_seq;
  a.seq_lens = pr->seq_lens;
  a.qsl = pr->query_start_loc;
  a.num_seqs = pr->num_seqs;
  a.block_size = pr->block_size;
  a.min_shared_pages = min_shared_pages;
  // a 16-column prefix pass must hold two members
  a.enabled = (pr->num_q_heads / pr->num_kv_heads) <= 8;
  a.plan = static_cast<int32_t*>(plan);
  const int e = ps_launch_cascade_plan(a, static_cast<cudaStream_t>(stream));
  if (e != 0) return cuda_fail(static_cast<cudaError_t>(e), "cascade plan launch");
  return PS_OK;
}

int64_t ps_paged_decode_cascade_workspace_size(int32_t num_seqs, int32_t num_q_heads,
                                               int32_t num_kv_heads, int32_t head_size) {
  if (num_seqs < 0 || num_seqs > ps::kCascadeMaxSeqs || num_kv_heads <= 0 || num_q_heads <= 0 ||
      head_size != 128) {
    fail(PS_ERR_INVALID_ARGUMENT, "workspace size: bad shape");
    return -1;
  }
  const int sms = sm_count_current(nullptr);
  if (sms <= 0) {
    fail(PS_ERR_CUDA, "no CUDA device");
    return -1;
  }
  return decode_layout(num_seqs, num_q_heads, num_kv_heads, sms, true).total;
}

int ps_paged_decode_cascade(const ps_paged_problem* pr, const void* plan, int64_t plan_bytes,
                            void* workspace, int64_t workspace_bytes, void* stream) {
  return decode_impl(pr, plan, plan_bytes, workspace, workspace_bytes, stream, true);
}

int ps_rope_kv_append(const ps_rope_append_problem* pr, void* stream) {
  if (!pr) return fail(PS_ERR_INVALID_ARGUMENT, "problem is NULL");
  if (pr->num_tokens < 0) return fail(PS_ERR_INVALID_ARGUMENT, "num_tokens < 0");
  if (pr->num_tokens == 0) return PS_OK;
  if (!pr->query || !pr->key || !pr->value || !pr->key_cache || !pr->value_cache ||
      !pr->slot_mapping || !pr->positions || !pr->cos_sin_cache)
    return fail(PS_ERR_INVALID_ARGUMENT, "a required pointer is NULL");
  if (pr->dtype != PS_DTYPE_BF16 && pr->dtype != PS_DTYPE_FP16)
    return fail(PS_ERR_UNSUPPORTED, "rope_kv_append supports fp16 and bf16 (dtype %d)", pr->dtype);
  if (pr->cos_sin_dtype != PS_DTYPE_FP32 && pr->cos_sin_dtype != pr->dtype)
    return fail(PS_ERR_UNSUPPORTED, "cos_sin_cache must be fp32 or the model dtype");
  if (pr->head_size <= 0 || pr->rotary_dim <= 0 || pr->rotary_dim % 2 || pr->rotary_dim > pr->head_size)
    return fail(PS_ERR_INVALID_ARGUMENT, "rotary_dim %d must be even and <= head_size %d",
                pr->rotary_dim, pr->head_size);
  if (pr->num_q_heads <= 0 || pr->num_kv_heads <= 0 || pr->block_size <= 0 || pr->num_blocks <= 0 ||
      pr->max_position <= 0 || pr->cos_sin_stride < pr->rotary_dim)
    return fail(PS_ERR_INVALID_ARGUMENT, "non-positive shape or cos_sin_stride < rotary_dim");
  int dev = 0;
  const int sms = sm_count_current(&dev);
  if (sms <= 0) return fail(PS_ERR_CUDA, "no CUDA device");
  const int es = 2;
  ps::RopeArgs a;
  a.q = static_cast<char*>(pr->query);
  a.q_st = pr->query_stride_token * es;
  a.q_sh = pr->query_stride_head * es;
  a.k = static_cast<char*>(pr->key);
  a.k_st = pr->key_stride_token * es;
  a.k_sh = pr->key_stride_head * es;
  a.v = static_cast<const char*>(pr->value);
  a.v_st = pr->value_stride_token * es;
  a.v_sh = pr->value_stride_head * es;
  a.key_cache = static_cast<char*>(pr->key_cache);
  a.value_cache = static_cast<char*>(pr->value_cache);
  a.c_sblock = pr->cache_stride_block * es;
  a.c_sslot = pr->cache_stride_slot * es;
  a.c_shead = pr->cache_stride_head * es;
  a.num_slots = pr->num_blocks * pr->block_size;
  a.block_size = pr->block_size;
  a.slot_mapping = pr->slot_mapping;
  a.positions = pr->positions;
  a.cos_sin = static_cast<const char*>(pr->cos_sin_cache);
  a.cs_fp32 = pr->cos_sin_dtype == PS_DTYPE_FP32;
  a.cs_stride_bytes = pr->cos_sin_stride * (a.cs_fp32 ? 4 : 2);
  a.max_position = pr->max_position;
  a.rotary_dim = pr->rotary_dim;
  a.neox = pr->is_neox != 0;
  a.num_tokens = pr->num_tokens;
  a.num_q_heads = pr->num_q_heads;
  a.num_kv_heads = pr->num_kv_heads;
  a.head_size = pr->head_size;
  a.bf16 = pr->dtype == PS_DTYPE_BF16;
  a.status = pr->status;
  // the 16-byte path needs every row and cos/sin row 16-byte aligned
  const int64_t cs_es = a.cs_fp32 ? 4 : 2;
  const bool vec = pr->head_size % 8 == 0 && pr->rotary_dim % 16 == 0 && aligned(pr->query, 16) &&
                   aligned(pr->key, 16) && aligned(pr->value, 16) && aligned(pr->key_cache, 16) &&
                   aligned(pr->value_cache, 16) && aligned(pr->cos_sin_cache, 16) &&
                   a.q_st % 16 == 0 && a.q_sh % 16 == 0 && a.k_st % 16 == 0 && a.k_sh % 16 == 0 &&
                   a.v_st % 16 == 0 && a.v_sh % 16 == 0 && a.c_sblock % 16 == 0 &&
                   a.c_sslot % 16 == 0 && a.c_shead % 16 == 0 && (pr->cos_sin_stride * cs_es) % 16 == 0 &&
                   (static_cast<const char*>(pr->value_cache) - static_cast<const char*>(pr->key_cache)) % 16 == 0;
  const int e = ps_launch_rope_kv_append(a, sms, vec ? 1 : 0, static_cast<cudaStream_t>(stream));
  if (e != 0) return cuda_fail(static_cast<cudaError_t>(e), "rope_kv_append launch");
  return PS_OK;
}

int ps_chunked_prefill(const ps_paged_problem* pr, void* stream) {
  return ps_chunked_prefill_ws(pr, nullptr, 0, stream);
}

int ps_chunked_prefill_ws(const ps_paged_problem* pr, void* workspace, int64_t workspace_bytes,
                          void* stream) {
  if (workspace != nullptr && (workspace_bytes < 256 || !aligned(workspace, 256)))
    return fail(PS_ERR_WORKSPACE, "prefill workspace must be >= 256 bytes, 256-byte aligned");
  int rc = validate_problem(pr, false);
  if (rc != PS_OK) return rc;
  if (pr->kv_cache_dtype != PS_KV_AUTO)
    return fail(PS_ERR_UNSUPPORTED, "chunked prefill over an fp8 cache is not built");
  if (pr->num_seqs == 0 || pr->num_tokens == 0) return PS_OK;
  if (pr->num_tokens < 0 || pr->num_tokens > INT32_MAX)
    return fail(PS_ERR_INVALID_ARGUMENT, "num_tokens out of range");
  if (pr->num_seqs > ps::kPrefillMaxSeqs)
    return fail(PS_ERR_UNSUPPORTED, "num_seqs %d > %d per prefill launch", pr->num_seqs,
                ps::kPrefillMaxSeqs);
  const int sms = sm_count_current(nullptr);
  if (sms <= 0) return fail(PS_ERR_CUDA, "no CUDA device");
  const int group = pr->num_q_heads / pr->num_kv_heads;
  const int tpt = 128 / group;
  CUtensorMap qmap, kmap, vmap;
  rc = make_q_map(&qmap, pr->q, pr->num_tokens, pr->num_q_heads, pr->q_stride_token,
                  pr->q_stride_head, group, tpt);
  if (rc != PS_OK) return rc;
  rc = make_page_map(&kmap, pr->key_cache, pr->num_blocks, pr->block_size, pr->num_kv_heads,
                     pr->cache_stride_block, pr->cache_stride_slot, pr->cache_stride_head);
  if (rc != PS_OK) return rc;
  rc = make_page_map(&vmap, pr->value_cache, pr->num_blocks, pr->block_size, pr->num_kv_heads,
                     pr->cache_stride_block, pr->cache_stride_slot, pr->cache_stride_head);
  if (rc != PS_OK) return rc;
  ps::PrefillParams p;
  p.block_table = pr->block_table;
  p.bt_stride = pr->block_table_stride;
  p.max_blocks_per_seq = pr->max_blocks_per_seq;
  p.seq_lens = pr->seq_lens;
  p.qsl = pr->query_start_loc;
  p.num_seqs = pr->num_seqs;
  p.out = pr->out;
  p.o_st = pr->out_stride_token;
  p.o_sh = pr->out_stride_head;
  p.lse = pr->lse;
  p.lse_sh = pr->lse_stride_head;
  p.lse_st = pr->lse_stride_token;
  p.num_q_heads = pr->num_q_heads;
  p.num_kv_heads = pr->num_kv_heads;
  p.group = group;
  p.tokens_per_tile = tpt;
  p.block_size = pr->block_size;
  p.num_blocks = pr->num_blocks;
  p.scale_log2 = pr->softmax_scale * 1.4426950408889634f;
  p.k_scale = pr->k_scale;
  p.v_scale = pr->v_scale;
  p.status = pr->status;
  // dynamic unit scheduling: two counters in the workspace's reserved header
  // (bytes 16..23; the decode uses bytes 0..3 of the same header)
  p.sched = workspace != nullptr ? reinterpret_cast<int32_t*>(static_cast<char*>(workspace) + 16) : nullptr;
  const int e = ps_launch_chunked_prefill(p, qmap, kmap, vmap, pr->dtype == PS_DTYPE_BF16, sms,
                                          static_cast<cudaStream_t>(stream));
  if (e != 0) return cuda_fail(static_cast<cudaError_t>(e), "chunked_prefill launch");
  return PS_OK;
}

}  // extern "C"

// ------------------------------------------------------------ DCP
// Slab layout: see dcp.cu.  Offsets depend only on (max_tokens, hq_local,
// world), which every rank of a group passes identically.
namespace {
struct DcpLayout {
  int64_t off_q, off_part, off_lse, off_qall, off_lens, total;
};
DcpLayout dcp_layout(int64_t max_tokens, int64_t hq_local, int64_t world) {
  const int64_t hq_all = hq_local * world;
  DcpLayout l;
  l.off_q = 256;
  l.off_part = round_up(l.off_q + max_tokens * hq_local * 256, 256);
  l.off_lse = round_up(l.off_part + max_tokens * hq_all * 256, 256);
  l.off_qall = round_up(l.off_lse + hq_all * max_tokens * 4, 256);
  l.off_lens = round_up(l.off_qall + max_tokens * hq_all * 256, 256);
  l.total = round_up(l.off_lens + max_tokens * 4, 256);
  return l;
}

// phase -1: the whole step; 0..4: one phase (ps_dcp_decode_phase)
int dcp_impl(const ps_dcp_problem* dp, int phase, void* workspace, int64_t workspace_bytes,
             void* stream) {
  if (!dp) return fail(PS_ERR_INVALID_ARGUMENT, "problem is NULL");
  if (phase < -1 || phase > 4) return fail(PS_ERR_INVALID_ARGUMENT, "phase %d outside [0, 4]", phase);
  const ps_paged_problem& lp = dp->local;
  if (dp->world < 1 || dp->world > PS_DCP_MAX_WORLD || dp->rank < 0 || dp->rank >= dp->world)
    return fail(PS_ERR_INVALID_ARGUMENT, "world %d / rank %d invalid (world <= %d)", dp->world,
                dp->rank, PS_DCP_MAX_WORLD);
  if (dp->interleave < 1 || lp.block_size % dp->interleave != 0)
    return fail(PS_ERR_INVALID_ARGUMENT, "interleave %d must divide block_size %d", dp->interleave,
                lp.block_size);
  if (dp->max_tokens < 1 || dp->max_tokens > ps::kDecodeMaxSeqs)
    return fail(PS_ERR_INVALID_ARGUMENT, "max_tokens %d outside [1, %d]", dp->max_tokens,
                ps::kDecodeMaxSeqs);
  for (int r = 0; r < dp->world; ++r)
    if (!dp->slabs[r] || !aligned(dp->slabs[r], 256))
      return fail(PS_ERR_INVALID_ARGUMENT, "slab of rank %d is NULL or not 256-byte aligned", r);
  if (lp.num_seqs < 0 || lp.num_seqs > dp->max_tokens)
    return fail(PS_ERR_INVALID_ARGUMENT, "num_seqs %d outside [0, max_tokens %d]", lp.num_seqs,
                dp->max_tokens);
  if (lp.query_start_loc != nullptr || lp.num_tokens != lp.num_seqs)
    return fail(PS_ERR_INVALID_ARGUMENT,
                "DCP decode takes one query row per sequence (query_start_loc NULL, num_tokens = num_seqs)");
  const int hq_local = lp.num_q_heads;
  if (hq_local <= 0) return fail(PS_ERR_INVALID_ARGUMENT, "num_q_heads must be positive");
  ps_paged_problem g = lp;  // the group's attention problem
  g.num_q_heads = hq_local * dp->world;
  int rc = validate_problem(&g, true);
  if (rc != PS_OK) return rc;
  if (lp.kv_cache_dtype != PS_KV_AUTO || lp.k_scale || lp.v_scale)
    return fail(PS_ERR_UNSUPPORTED, "DCP decode over an fp8 or scaled cache is not built");
  const bool context_only = (dp->flags & PS_DCP_CONTEXT_ONLY) != 0;
  if (dp->flags & ~PS_DCP_CONTEXT_ONLY) return fail(PS_ERR_INVALID_ARGUMENT, "unknown DCP flags");
  if (!context_only) {
    if (!lp.new_key || !lp.new_value || !lp.slot_mapping)
      return fail(PS_ERR_INVALID_ARGUMENT, "DCP decode needs new_key, new_value and slot_mapping");
    if (!aligned(lp.new_key, 16) || !aligned(lp.new_value, 16) || lp.new_key_stride_token % 8 ||
        lp.new_key_stride_head % 8 || lp.new_value_stride_token % 8 || lp.new_value_stride_head % 8)
      return fail(PS_ERR_INVALID_ARGUMENT, "new key/value rows must be 16-byte aligned");
  }
  if (!workspace || !aligned(workspace, 256))
    return fail(PS_ERR_WORKSPACE, "DCP decode needs a 256-byte aligned decode workspace");
  if (lp.num_seqs == 0) return PS_OK;
  int dev = 0;
  const int sms = sm_count_current(&dev);
  if (sms <= 0) return fail(PS_ERR_CUDA, "no CUDA device");
  const DcpLayout lay = dcp_layout(dp->max_tokens, hq_local, dp->world);
  char* own = static_cast<char*>(dp->slabs[dp->rank]);
  const int64_t eb = 2;
  ps::DcpArgs a;
  a.world = dp->world;
  a.rank = dp->rank;
  a.interleave = dp->interleave;
  for (int r = 0; r < ps::kDcpMaxWorld; ++r)
    a.slab[r] = r < dp->world ? static_cast<char*>(dp->slabs[r]) : nullptr;
  a.off_q = lay.off_q;
  a.off_part = lay.off_part;
  a.off_lse = lay.off_lse;
  a.off_qall = lay.off_qall;
  a.off_lens = lay.off_lens;
  a.signal_first = phase == -1 ? 1 : 0;
  a.context_only = context_only ? 1 : 0;
  a.q = static_cast<const char*>(lp.q);
  a.q_st = lp.q_stride_token * eb;
  a.q_sh = lp.q_stride_head * eb;
  a.out = static_cast<char*>(lp.out);
  a.o_st = lp.out_stride_token * eb;
  a.o_sh = lp.out_stride_head * eb;
  a.lse = lp.lse;
  a.lse_sh = lp.lse_stride_head;
  a.lse_st = lp.lse_stride_token;
  a.new_key = static_cast<const char*>(lp.new_key);
  a.nk_st = lp.new_key_stride_token * eb;
  a.nk_sh = lp.new_key_stride_head * eb;
  a.new_value = static_cast<const char*>(lp.new_value);
  a.nv_st = lp.new_value_stride_token * eb;
  a.nv_sh = lp.new_value_stride_head * eb;
  a.slot_mapping = lp.slot_mapping;
  a.key_cache = static_cast<char*>(const_cast<void*>(lp.key_cache));
  a.value_cache = static_cast<char*>(const_cast<void*>(lp.value_cache));
  a.c_sblock = lp.cache_stride_block * eb;
  a.c_sslot = lp.cache_stride_slot * eb;
  a.c_shead = lp.cache_stride_head * eb;
  a.num_slots = lp.num_blocks * lp.block_size;
  a.block_size = lp.block_size;
  a.seq_lens = lp.seq_lens;
  a.num_tokens = lp.num_seqs;
  a.hq_local = hq_local;
  a.hq_all = g.num_q_heads;
  a.num_kv_heads = lp.num_kv_heads;
  a.group = g.num_q_heads / lp.num_kv_heads;
  a.softmax_scale = lp.softmax_scale;
  a.bf16 = lp.dtype == PS_DTYPE_BF16 ? 1 : 0;
  a.status = static_cast<int32_t*>(workspace);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto launch = [&](int which) -> int {
    const int e = ps_launch_dcp(a, which, sms, s);
    return e != 0 ? cuda_fail(static_cast<cudaError_t>(e), "dcp launch") : PS_OK;
  };
  auto attend_local = [&]() -> int {
    // plain decode of the group's heads over this rank's slice; partial
    // outputs and LSEs into the slab, no fused append
    ps_paged_problem d = g;
    d.q = own + lay.off_qall;
    d.q_stride_token = static_cast<int64_t>(g.num_q_heads) * 128;
    d.q_stride_head = 128;
    d.seq_lens = reinterpret_cast<const int32_t*>(own + lay.off_lens);
    d.out = own + lay.off_part;
    d.out_stride_token = static_cast<int64_t>(g.num_q_heads) * 128;
    d.out_stride_head = 128;
    d.lse = reinterpret_cast<float*>(own + lay.off_lse);
    d.lse_stride_head = lp.num_seqs;
    d.lse_stride_token = 1;
    d.new_key = nullptr;
    d.new_value = nullptr;
    d.slot_mapping = nullptr;
    return decode_impl(&d, nullptr, 0, workspace, workspace_bytes, stream, false);
  };
  switch (phase) {
    case -1:
      if ((rc = launch(0)) != PS_OK || (rc = launch(2)) != PS_OK || (rc = attend_local()) != PS_OK)
        return rc;
      return launch(4);
    case 2:
      if ((rc = launch(2)) != PS_OK) return rc;
      return attend_local();
    default:
      return launch(phase);
  }
}
}  // namespace

extern "C" {

int64_t ps_dcp_slab_bytes(int32_t max_tokens, int32_t hq_local, int32_t world) {
  if (max_tokens < 1 || max_tokens > ps::kDecodeMaxSeqs || hq_local < 1 || world < 1 ||
      world > PS_DCP_MAX_WORLD) {
    fail(PS_ERR_INVALID_ARGUMENT, "slab size: bad shape");
    return -1;
  }
  return dcp_layout(max_tokens, hq_local, world).total;
}

int ps_dcp_slab_alloc(int64_t bytes, void** slab) {
  if (!slab || bytes <= 0) return fail(PS_ERR_INVALID_ARGUMENT, "slab alloc: bad arguments");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, static_cast<size_t>(bytes));
  if (e != cudaSuccess) return cuda_fail(e, "slab cudaMalloc");
  e = cudaMemset(p, 0, static_cast<size_t>(bytes));
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_fail(e, "slab zeroing");
  }
  *slab = p;
  return PS_OK;
}

int ps_dcp_slab_free(void* slab) {
  if (!slab) return PS_OK;
  const cudaError_t e = cudaFree(slab);
  return e == cudaSuccess ? PS_OK : cuda_fail(e, "slab cudaFree");
}

int ps_dcp_ipc_handle(const void* slab, void* handle) {
  if (!slab || !handle) return fail(PS_ERR_INVALID_ARGUMENT, "ipc handle: NULL argument");
  static_assert(sizeof(cudaIpcMemHandle_t) == PS_DCP_IPC_HANDLE_BYTES, "IPC handle size");
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(slab));
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcGetMemHandle");
  std::memcpy(handle, &h, sizeof(h));
  return PS_OK;
}

int ps_dcp_ipc_open(const void* handle, void** peer_slab) {
  if (!handle || !peer_slab) return fail(PS_ERR_INVALID_ARGUMENT, "ipc open: NULL argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(peer_slab, h, cudaIpcMemLazyEnablePeerAccess);
  return e == cudaSuccess ? PS_OK : cuda_fail(e, "cudaIpcOpenMemHandle");
}

int ps_dcp_ipc_close(void* peer_slab) {
  if (!peer_slab) return PS_OK;
  const cudaError_t e = cudaIpcCloseMemHandle(peer_slab);
  return e == cudaSuccess ? PS_OK : cuda_fail(e, "cudaIpcCloseMemHandle");
}

int ps_dcp_decode(const ps_dcp_problem* problem, void* workspace, int64_t workspace_bytes,
                  void* stream) {
  return dcp_impl(problem, -1, workspace, workspace_bytes, stream);
}

int ps_dcp_decode_phase(const ps_dcp_problem* problem, int32_t phase, void* workspace,
                        int64_t workspace_bytes, void* stream) {
  return dcp_impl(problem, phase, workspace, workspace_bytes, stream);
}

}  // extern "C"

// ------------------------------------------------------------ head gather
namespace {
int validate_gather(const ps_head_gather_problem* hp) {
  if (!hp) return fail(PS_ERR_INVALID_ARGUMENT, "problem is NULL");
  if (hp->world < 1 || hp->world > PS_DCP_MAX_WORLD || hp->rank < 0 || hp->rank >= hp->world)
    return fail(PS_ERR_INVALID_ARGUMENT, "world %d / rank %d invalid (world <= %d)", hp->world, hp->rank,
                PS_DCP_MAX_WORLD);
  if (hp->max_tokens < 1 || hp->num_tokens < 0 || hp->num_tokens > hp->max_tokens || hp->hq_local < 1)
    return fail(PS_ERR_INVALID_ARGUMENT, "num_tokens %d / max_tokens %d / hq_local %d invalid",
                hp->num_tokens, hp->max_tokens, hp->hq_local);
  if (hp->dtype != PS_DTYPE_BF16 && hp->dtype != PS_DTYPE_FP16)
    return fail(PS_ERR_UNSUPPORTED, "head gather moves 2-byte rows (dtype %d)", hp->dtype);
  for (int r = 0; r < hp->world; ++r)
    if (!hp->slabs[r] || !aligned(hp->slabs[r], 256))
      return fail(PS_ERR_INVALID_ARGUMENT, "slab of rank %d is NULL or not 256-byte aligned", r);
  if (!hp->out || !aligned(hp->out, 16) || hp->out_stride_token % 8 || hp->out_stride_head % 8)
    return fail(PS_ERR_INVALID_ARGUMENT, "out base/strides must be 16-byte aligned");
  if (!hp->status) return fail(PS_ERR_INVALID_ARGUMENT, "head gather needs a device status word");
  return PS_OK;
}

int head_gather_impl(const ps_head_gather_problem* hp, int which, void* stream) {
  const int rc = validate_gather(hp);
  if (rc != PS_OK) return rc;
  if (hp->num_tokens == 0) return PS_OK;
  const int sms = sm_count_current(nullptr);
  if (sms <= 0) return fail(PS_ERR_CUDA, "no CUDA device");
  ps::HeadGatherArgs a;
  a.world = hp->world;
  a.rank = hp->rank;
  for (int r = 0; r < ps::kDcpMaxWorld; ++r)
    a.slab[r] = r < hp->world ? static_cast<char*>(hp->slabs[r]) : nullptr;
  a.num_tokens = hp->num_tokens;
  a.hq_local = hp->hq_local;
  a.out = static_cast<char*>(hp->out);
  a.o_st = hp->out_stride_token * 2;
  a.o_sh = hp->out_stride_head * 2;
  a.status = hp->status;
  a.mode = 0;
  const int e = ps_launch_head_gather(a, which, sms, static_cast<cudaStream_t>(stream));
  return e != 0 ? cuda_fail(static_cast<cudaError_t>(e), "head gather launch") : PS_OK;
}
}  // namespace

extern "C" {

int64_t ps_head_gather_slab_bytes(int32_t max_tokens, int32_t hq_local) {
  if (max_tokens < 1 || hq_local < 1) {
    fail(PS_ERR_INVALID_ARGUMENT, "head gather slab size: bad shape");
    return -1;
  }
  return round_up(PS_HEAD_GATHER_ROWS_OFFSET + static_cast<int64_t>(max_tokens) * hq_local * 256, 256);
}

int ps_head_gather(const ps_head_gather_problem* problem, void* stream) {
  return head_gather_impl(problem, 0, stream);
}

int64_t ps_decode_head_gather_slab_bytes(int32_t max_tokens, int32_t num_q_heads) {
  if (max_tokens < 1 || num_q_heads < 1) {
    fail(PS_ERR_INVALID_ARGUMENT, "decode head gather slab size: bad shape");
    return -1;
  }
  return round_up(ps::kDecodeGatherRowsOffset + static_cast<int64_t>(max_tokens) * num_q_heads * 256, 256);
}

int ps_paged_decode_head_gather(const ps_paged_problem* problem, void* workspace, int64_t workspace_bytes,
                                const ps_head_gather_problem* gather, void* stream) {
  int rc = validate_gather(gather);
  if (rc != PS_OK) return rc;
  if (!problem) return fail(PS_ERR_INVALID_ARGUMENT, "problem is NULL");
  if (problem->num_q_heads != gather->hq_local)
    return fail(PS_ERR_INVALID_ARGUMENT, "problem's %d query heads != the gather's hq_local %d",
                problem->num_q_heads, gather->hq_local);
  if (problem->dtype != gather->dtype)
    return fail(PS_ERR_INVALID_ARGUMENT, "problem dtype %d != gather dtype %d", problem->dtype, gather->dtype);
  if (problem->num_seqs > gather->num_tokens)
    return fail(PS_ERR_INVALID_ARGUMENT, "%d sequences > the gather's %d tokens", problem->num_seqs,
                gather->num_tokens);
  if (gather->num_tokens == 0 || problem->num_seqs == 0)
    return fail(PS_ERR_INVALID_ARGUMENT, "an empty step has no rows to gather (every rank must skip it)");
  // this rank's heads of the group's output
  ps_paged_problem local = *problem;
  local.out = static_cast<char*>(gather->out) +
              static_cast<int64_t>(gather->rank) * gather->hq_local * gather->out_stride_head * 2;
  local.out_stride_token = gather->out_stride_token;
  local.out_stride_head = gather->out_stride_head;
  return decode_impl(&local, nullptr, 0, workspace, workspace_bytes, stream, false, gather);
}

int ps_head_gather_phase(const ps_head_gather_problem* problem, int32_t phase, void* stream) {
  if (phase < 0 || phase > 2) return fail(PS_ERR_INVALID_ARGUMENT, "phase %d outside [0, 2]", phase);
  return head_gather_impl(problem, phase + 1, stream);  // launcher: 1 signal, 2 pull, 3 finish
}

}  // extern "C"

extern "C" int ps_kv_dequant_gather(const ps_paged_problem* pr, int32_t max_pages, void* out_key,
                                    void* out_value, void* stream) {
  if (!pr) return fail(PS_ERR_INVALID_ARGUMENT, "problem is NULL");
  if (pr->kv_cache_dtype != PS_KV_FP8_E4M3)
    return fail(PS_ERR_INVALID_ARGUMENT, "dequantizing gather reads an fp8 cache");
  if (pr->num_seqs < 0 || max_pages < 0) return fail(PS_ERR_INVALID_ARGUMENT, "negative shape");
  if (pr->num_seqs == 0 || max_pages == 0) return PS_OK;
  if (!pr->key_cache || !pr->value_cache || !pr->block_table || !pr->seq_lens || !out_key || !out_value)
    return fail(PS_ERR_INVALID_ARGUMENT, "a required pointer is NULL");
  if (pr->dtype != PS_DTYPE_BF16 && pr->dtype != PS_DTYPE_FP16)
    return fail(PS_ERR_UNSUPPORTED, "scratch dtype must be fp16 or bf16 (dtype %d)", pr->dtype);
  if (pr->head_size != 128 || pr->num_kv_heads <= 0 || pr->block_size <= 0 || pr->block_size % 16)
    return fail(PS_ERR_INVALID_ARGUMENT, "shape: head_size 128, block_size a multiple of 16");
  if (pr->cache_stride_head != 128 || pr->cache_stride_slot != static_cast<int64_t>(pr->num_kv_heads) * 128 ||
      pr->cache_stride_block % 16 || !aligned(pr->key_cache, 16) || !aligned(pr->value_cache, 16))
    return fail(PS_ERR_INVALID_ARGUMENT, "fp8 cache blocks must be contiguous and 16-byte aligned");
  if (!aligned(out_key, 16) || !aligned(out_value, 16))
    return fail(PS_ERR_INVALID_ARGUMENT, "scratch must be 16-byte aligned");
  if (pr->block_table_stride < pr->max_blocks_per_seq)
    return fail(PS_ERR_INVALID_ARGUMENT, "block_table_stride < max_blocks_per_seq");
  const int sms = sm_count_current(nullptr);
  if (sms <= 0) return fail(PS_ERR_CUDA, "no CUDA device");
  ps::DequantArgs a;
  a.key_cache = static_cast<const char*>(pr->key_cache);
  a.value_cache = static_cast<const char*>(pr->value_cache);
  a.c_sblock = pr->cache_stride_block;
  a.block_bytes = static_cast<int64_t>(pr->block_size) * pr->num_kv_heads * 128;
  a.num_blocks = pr->num_blocks;
  a.block_table = pr->block_table;
  a.bt_stride = pr->block_table_stride;
  a.max_blocks_per_seq = pr->max_blocks_per_seq;
  a.seq_lens = pr->seq_lens;
  a.num_seqs = pr->num_seqs;
  a.max_pages = max_pages;
  a.block_size = pr->block_size;
  a.k_scale = pr->k_scale;
  a.v_scale = pr->v_scale;
  a.out_key = static_cast<char*>(out_key);
  a.out_value = static_cast<char*>(out_value);
  a.status = pr->status;
  const int e = ps_launch_kv_dequant_gather(a, pr->dtype == PS_DTYPE_BF16, sms,
                                            static_cast<cudaStream_t>(stream));
  return e != 0 ? cuda_fail(static_cast<cudaError_t>(e), "dequantizing gather launch") : PS_OK;
}

extern "C" int ps_merge_attn_states(const void* prefix_out, int64_t prefix_stride_token,
                                    int64_t prefix_stride_head, const float* prefix_lse,
                                    const void* suffix_out, int64_t suffix_stride_token,
                                    int64_t suffix_stride_head, const float* suffix_lse, void* out,
                                    int64_t out_stride_token, int64_t out_stride_head, float* out_lse,
                                    int64_t num_tokens, int32_t num_heads, int32_t head_size,
                                    int32_t dtype, void* stream) {
  if (num_tokens < 0 || num_heads < 0) return fail(PS_ERR_INVALID_ARGUMENT, "negative shape");
  if (num_tokens == 0 || num_heads == 0) return PS_OK;
  if (!prefix_out || !prefix_lse || !suffix_out || !suffix_lse || !out)
    return fail(PS_ERR_INVALID_ARGUMENT, "a required pointer is NULL");
  if (head_size != 128) return fail(PS_ERR_UNSUPPORTED, "head_size %d unsupported (128)", head_size);
  if (dtype != PS_DTYPE_BF16 && dtype != PS_DTYPE_FP16)
    return fail(PS_ERR_UNSUPPORTED, "merge takes fp16 or bf16 outputs (dtype %d)", dtype);
  const int64_t st[6] = {prefix_stride_token, prefix_stride_head, suffix_stride_token,
                         suffix_stride_head, out_stride_token, out_stride_head};
  for (int64_t x : st)
    if (x % 4) return fail(PS_ERR_INVALID_ARGUMENT, "output strides must be 8-byte aligned");
  if (!aligned(prefix_out, 8) || !aligned(suffix_out, 8) || !aligned(out, 8))
    return fail(PS_ERR_INVALID_ARGUMENT, "outputs must be 8-byte aligned");
  const int sms = sm_count_current(nullptr);
  if (sms <= 0) return fail(PS_ERR_CUDA, "no CUDA device");
  ps::MergeArgs a;
  a.p_out = static_cast<const char*>(prefix_out);
  a.p_st = prefix_stride_token * 2;
  a.p_sh = prefix_stride_head * 2;
  a.p_lse = prefix_lse;
  a.s_out = static_cast<const char*>(suffix_out);
  a.s_st = suffix_stride_token * 2;
  a.s_sh = suffix_stride_head * 2;
  a.s_lse = suffix_lse;
  a.out = static_cast<char*>(out);
  a.o_st = out_stride_token * 2;
  a.o_sh = out_stride_head * 2;
  a.out_lse = out_lse;
  a.num_tokens = num_tokens;
  a.num_heads = num_heads;
  const int e = ps_launch_merge_attn_states(a, dtype == PS_DTYPE_BF16, sms, static_cast<cudaStream_t>(stream));
  return e != 0 ? cuda_fail(static_cast<cudaError_t>(e), "merge launch") : PS_OK;
}
